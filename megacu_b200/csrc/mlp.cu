// Tensor-parallel MLP blocks (benchmark config 5, no counterpart in megacu):
//   act   = silu(x @ w_gate) * (x @ w_up)      column-parallel, local
//   x_out = allreduce_pe(act @ w_down)          row-parallel, fused exchange
// megacu_cuda_gemm_swiglu_bf16 is the first line as one persistent launch of
// the megakernel's SwiGLU variant; megacu_cuda_mlp_chain_bf16 runs `layers`
// such blocks back to back: either each block as one SwiGLU launch and one
// fused GEMM + allreduce launch (megacu_cuda_gemm_allreduce_bf16), the output
// of one block feeding the next, or all blocks (up to six) in one persistent
// launch of mlp_chain_megakernel, whose blocks wait for each other through
// counters in the event tensor.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include <megacu_b200.h>

#include "kernels/chain_kernel.cuh"
#include "kernels/gemm_ar_kernel.cuh"
#include "kernels/launch.cuh"
#include "team.h"
#include "tma_map.h"

namespace {

using namespace megacu_b200;

// The gate/up projection with the SiLU * up epilogue (one PE): `mg` and `mu`
// are the gate and up weights [k, n] with 64 x 64 boxes.
cudaError_t launch_swiglu(bool pairs, int device, int grid, cudaStream_t stream,
                          CUtensorMap const &ma, CUtensorMap const &mg, CUtensorMap const &mu,
                          gemm_ar_params const &prm) {
  return pairs ? launch_variant<256, false, true, true>(device, grid, stream, ma, mg, mu, prm)
               : launch_variant<256, false, false, true>(device, grid, stream, ma, mg, mu, prm);
}

constexpr std::int32_t kActTile = 128;  // act columns per tile (128 gate + 128 up)
constexpr std::int32_t kMaxLayers = 64;

megacu_status ok_status() { return {MEGACU_OK, 0, nullptr}; }

megacu_status fail(megacu_status_code code, std::uint16_t detail, char const *msg) {
  return {static_cast<std::uint8_t>(code), detail, msg};
}

megacu_status cuda_fail(cudaError_t e, std::uint16_t detail) {
  return {MEGACU_LAUNCH_ERROR, detail, cudaGetErrorString(e)};
}

struct swiglu_plan {
  std::int32_t m_tiles = 0, n_tiles = 0, tiles = 0;
  std::int32_t pairs = 0;
  std::int64_t events_bytes = 0;
};

// problem.m = tokens, problem.n = act columns (this PE's intermediate slice),
// problem.k = hidden.
megacu_status make_swiglu_plan(megacu_gemm_ar_problem_v2 const &p, swiglu_plan &out) {
  if (p.m <= 0 || p.n <= 0 || p.k <= 0) return fail(MEGACU_INVALID_ARGUMENT, 1, "invalid problem");
  if (p.dtype != MEGACU_DTYPE_BF16) return fail(MEGACU_UNSUPPORTED, 20, "SwiGLU needs dtype bf16");
  if (p.n % 8 != 0 || p.k % 8 != 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 21, "n and k must be multiples of 8 (16-byte rows)");
  }
  if (p.m > (1ll << 30) || p.n > (1ll << 30) || p.k > (1ll << 30)) {
    return fail(MEGACU_UNSUPPORTED, 22, "dimension too large");
  }
  if ((p.tile_m != 0 && p.tile_m != kBlockM) || (p.tile_n != 0 && p.tile_n != kActTile)) {
    return fail(MEGACU_UNSUPPORTED, 22, "SwiGLU tiles are 128 x 128 act columns");
  }
  if (p.cta_pairs < MEGACU_CTA_PAIRS_AUTO || p.cta_pairs > MEGACU_CTA_PAIRS_ON) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "unknown cta_pairs");
  }
  swiglu_plan pl;
  pl.m_tiles = static_cast<std::int32_t>((p.m + kBlockM - 1) / kBlockM);
  pl.n_tiles = static_cast<std::int32_t>((p.n + kActTile - 1) / kActTile);
  std::int64_t const tiles = static_cast<std::int64_t>(pl.m_tiles) * pl.n_tiles;
  if (tiles > (1 << 24)) return fail(MEGACU_UNSUPPORTED, 22, "too many tiles");
  pl.tiles = static_cast<std::int32_t>(tiles);
  tile_schedule const sched{pl.m_tiles, pl.n_tiles, 1, mode_allreduce, 16};
  bool const can_pair = pairs_fit(sched);
  if (p.cta_pairs == MEGACU_CTA_PAIRS_ON && !can_pair) {
    return fail(MEGACU_UNSUPPORTED, 27, "CTA pairs need an even number of tile rows");
  }
  pl.pairs = (can_pair && p.cta_pairs != MEGACU_CTA_PAIRS_OFF) ? 1 : 0;
  pl.events_bytes = events_bytes_for(1, pl.tiles);
  out = pl;
  return ok_status();
}

bool aligned16(void const *p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

megacu_status run_swiglu(megacu_driver_view driver, void const *x, void const *w_gate,
                         void const *w_up, void *act, void *events,
                         megacu_gemm_ar_problem_v2 problem) {
  swiglu_plan pl;
  megacu_status st = make_swiglu_plan(problem, pl);
  if (st.code != MEGACU_OK) return st;
  if (x == nullptr || w_gate == nullptr || w_up == nullptr || act == nullptr || events == nullptr) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  if (!aligned16(x) || !aligned16(w_gate) || !aligned16(w_up) || !aligned16(act) ||
      !aligned16(events)) {
    return fail(MEGACU_INVALID_ARGUMENT, 21, "buffers must be 16-byte aligned");
  }
  if (driver.launch.stream == nullptr) return ok_status();
  int const device = driver.launch.device_ordinal;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  CUtensorMap map_x, map_g, map_u;
  if (!encode_bf16_map(&map_x, x, problem.m, problem.k, kBlockM) ||
      !encode_bf16_map(&map_g, w_gate, problem.k, problem.n, kBlockK) ||
      !encode_bf16_map(&map_u, w_up, problem.k, problem.n, kBlockK)) {
    return fail(MEGACU_BACKEND_ERROR, 30, "cuTensorMapEncodeTiled failed");
  }
  gemm_ar_params prm{};
  prm.m = static_cast<std::int32_t>(problem.m);
  prm.n = static_cast<std::int32_t>(problem.n);
  prm.k = static_cast<std::int32_t>(problem.k);
  prm.m_tiles = pl.m_tiles;
  prm.n_tiles = pl.n_tiles;
  prm.tiles = pl.tiles;
  prm.n_pes = 1;
  prm.my_pe = 0;
  prm.mode = mode_allreduce;
  prm.group_m = 16;
  prm.comm_warps = kWorkerWarps;  // unused with one PE
  prm.rows_per_pe = prm.m;
  prm.timeout_ns = problem.timeout_ns != 0 ? problem.timeout_ns : 10000000000ull;
  prm.out = static_cast<__nv_bfloat16 *>(act);
  prm.events = static_cast<std::uint32_t *>(events);
  prm.peers.n_pes = 1;
  prm.trace = reinterpret_cast<unsigned long long *>(problem.trace);
  prm.trace_capacity = problem.trace != nullptr ? problem.trace_capacity : 0;
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  int const grid = problem.num_ctas > 0 ? problem.num_ctas : sms;
  e = launch_swiglu(pl.pairs != 0, device, grid, static_cast<cudaStream_t>(driver.launch.stream),
                    map_x, map_g, map_u, prm);
  if (e != cudaSuccess) return cuda_fail(e, 14);
  return ok_status();
}

megacu_gemm_ar_problem_v2 swiglu_problem(megacu_mlp_chain_problem const &p) {
  megacu_gemm_ar_problem_v2 q{};
  q.m = p.tokens;
  q.n = p.inter;
  q.k = p.hidden;
  q.mode = MEGACU_MODE_ALLREDUCE;
  q.dtype = MEGACU_DTYPE_BF16;
  q.num_ctas = p.num_ctas;
  q.cta_pairs = p.cta_pairs;
  q.timeout_ns = p.timeout_ns;
  return q;
}

megacu_gemm_ar_problem_v2 down_problem(megacu_mlp_chain_problem const &p) {
  megacu_gemm_ar_problem_v2 q{};
  q.m = p.tokens;
  q.n = p.hidden;
  q.k = p.inter;
  q.mode = MEGACU_MODE_ALLREDUCE;
  q.algo = p.algo;
  q.deterministic = p.deterministic;
  q.dtype = MEGACU_DTYPE_BF16;
  q.num_ctas = p.num_ctas;
  q.cta_pairs = p.cta_pairs;
  q.timeout_ns = p.timeout_ns;
  return q;
}

// ---- the whole chain in one persistent launch ---------------------------------

static_assert(sizeof(chain_maps) + sizeof(chain_params) <= 4096, "kernel parameter space");

struct chain_plan {
  std::int32_t m_tiles = 0, gu_tiles_n = 0, dn_tiles_n = 0;
  std::int32_t pairs = 0;
  std::int64_t workspace_bytes = 0;  // one plane of partial slots
  std::int64_t events_bytes = 0;
};

megacu_status make_chain_plan(megacu_mlp_chain_problem const &p, std::int32_t n_pes,
                              chain_plan &out) {
  if (p.layers > kChainMaxLayers) {
    return fail(MEGACU_UNSUPPORTED, 29, "a single-launch chain holds at most 6 blocks");
  }
  if (p.deterministic) {
    return fail(MEGACU_UNSUPPORTED, 29, "a single-launch chain exchanges bf16 partials");
  }
  if (p.hidden % 8 != 0 || p.inter % 8 != 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 21, "hidden and inter must be multiples of 8");
  }
  if (p.tokens > (1ll << 30) || p.hidden > (1ll << 30) || p.inter > (1ll << 30)) {
    return fail(MEGACU_UNSUPPORTED, 22, "dimension too large");
  }
  if (n_pes < 1 || n_pes > megacu::nvshmem::max_team_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "team size must be 1..8");
  }
  if (p.cta_pairs < MEGACU_CTA_PAIRS_AUTO || p.cta_pairs > MEGACU_CTA_PAIRS_ON) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "unknown cta_pairs");
  }
  chain_plan pl;
  pl.m_tiles = static_cast<std::int32_t>((p.tokens + kBlockM - 1) / kBlockM);
  pl.gu_tiles_n = static_cast<std::int32_t>((p.inter + kChainActTile - 1) / kChainActTile);
  pl.dn_tiles_n = static_cast<std::int32_t>((p.hidden + kChainBN - 1) / kChainBN);
  if (static_cast<std::int64_t>(pl.m_tiles) * (pl.gu_tiles_n + pl.dn_tiles_n) > (1 << 24)) {
    return fail(MEGACU_UNSUPPORTED, 22, "too many tiles");
  }
  bool const can_pair = pl.m_tiles % 2 == 0;  // raster bands of 16 rows: even
  if (p.cta_pairs == MEGACU_CTA_PAIRS_ON && !can_pair) {
    return fail(MEGACU_UNSUPPORTED, 27, "CTA pairs need an even number of token blocks");
  }
  pl.pairs = (can_pair && p.cta_pairs != MEGACU_CTA_PAIRS_OFF) ? 1 : 0;
  pl.workspace_bytes = n_pes == 1 ? 0
                                  : static_cast<std::int64_t>(pl.m_tiles) * pl.dn_tiles_n *
                                        kBlockM * kChainBN * 2;
  pl.events_bytes = chain_events_bytes(p.layers, n_pes, pl.dn_tiles_n, pl.m_tiles);
  out = pl;
  return ok_status();
}

megacu_status run_chain_single_launch(megacu_driver_view driver, void const *x,
                                      void const *const *w_gate, void const *const *w_up,
                                      void const *const *w_down, void *act, void *workspace,
                                      void *x_work, void *out, void *events,
                                      megacu_mlp_chain_problem const &problem) {
  std::int32_t const n_pes = driver.team.team_n_pes;
  std::int32_t const my_pe = driver.team.team_my_pe;
  chain_plan pl;
  megacu_status st = make_chain_plan(problem, n_pes, pl);
  if (st.code != MEGACU_OK) return st;
  if (my_pe < 0 || my_pe >= n_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "team_my_pe out of range");
  }
  if (x == nullptr || act == nullptr || events == nullptr || (n_pes > 1 && workspace == nullptr)) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  void const *all[] = {x, act, x_work, out, events};
  for (void const *ptr : all) {
    if (!aligned16(ptr)) return fail(MEGACU_INVALID_ARGUMENT, 21, "buffers must be 16-byte aligned");
  }
  for (std::int32_t l = 0; l < problem.layers; ++l) {
    if (w_gate[l] == nullptr || w_up[l] == nullptr || w_down[l] == nullptr) {
      return fail(MEGACU_INVALID_ARGUMENT, 2, "missing weights");
    }
    if (!aligned16(w_gate[l]) || !aligned16(w_up[l]) || !aligned16(w_down[l])) {
      return fail(MEGACU_INVALID_ARGUMENT, 21, "buffers must be 16-byte aligned");
    }
  }
  team_impl *team = nullptr;
  std::int64_t const x_bytes = problem.tokens * problem.hidden * 2;
  if (n_pes > 1) {
    team = as_team(driver.team.team);
    if (team == nullptr) {
      return fail(MEGACU_UNSUPPORTED, 13, "remote PEs need a megacu_b200 team in team_view.team");
    }
    if (!team->connected || team->n_pes != n_pes || team->my_pe != my_pe) {
      return fail(MEGACU_INVALID_ARGUMENT, 24, "team handle does not match team_view");
    }
    if (!team->contains(workspace, pl.workspace_bytes) ||
        !team->contains(events, pl.events_bytes) || !team->contains(out, x_bytes) ||
        !team->contains(x_work, x_bytes)) {
      return fail(MEGACU_INVALID_ARGUMENT, 25,
                  "workspace, events, out and x_work must lie in the team's symmetric heap");
    }
  }
  if (driver.launch.stream == nullptr) return ok_status();
  int const device = driver.launch.device_ordinal;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  if (team != nullptr && team->device != device) {
    return fail(MEGACU_INVALID_ARGUMENT, 24, "team was created on another device");
  }

  chain_maps maps{};
  bool ok = encode_bf16_map(&maps.map[kChainMapX], x, problem.tokens, problem.hidden, kBlockM) &&
            encode_bf16_map(&maps.map[kChainMapOut], out, problem.tokens, problem.hidden, kBlockM) &&
            encode_bf16_map(&maps.map[kChainMapWork], x_work, problem.tokens, problem.hidden,
                            kBlockM) &&
            encode_bf16_map(&maps.map[kChainMapAct], act, problem.tokens, problem.inter, kBlockM);
  for (std::int32_t l = 0; ok && l < problem.layers; ++l) {
    CUtensorMap *m = &maps.map[kChainMapLayer0 + 3 * l];
    ok = encode_bf16_map(m + 0, w_gate[l], problem.hidden, problem.inter, kBlockK) &&
         encode_bf16_map(m + 1, w_up[l], problem.hidden, problem.inter, kBlockK) &&
         encode_bf16_map(m + 2, w_down[l], problem.inter, problem.hidden, kBlockK);
  }
  if (!ok) return fail(MEGACU_BACKEND_ERROR, 30, "cuTensorMapEncodeTiled failed");

  chain_params prm{};
  prm.tokens = static_cast<std::int32_t>(problem.tokens);
  prm.hidden = static_cast<std::int32_t>(problem.hidden);
  prm.inter = static_cast<std::int32_t>(problem.inter);
  prm.layers = problem.layers;
  prm.m_tiles = pl.m_tiles;
  prm.gu_tiles_n = pl.gu_tiles_n;
  prm.dn_tiles_n = pl.dn_tiles_n;
  prm.gu_units = pl.m_tiles * pl.gu_tiles_n / (pl.pairs ? 2 : 1);
  prm.dn_units = pl.m_tiles * pl.dn_tiles_n / (pl.pairs ? 2 : 1);
  prm.n_pes = n_pes;
  prm.my_pe = my_pe;
  prm.group_m = 16;
  tile_schedule const sched_dn{pl.m_tiles, pl.dn_tiles_n, n_pes, mode_allreduce, 16};
  prm.n_comm = n_pes == 1 ? 0 : owned_tiles(sched_dn, my_pe) * kQuarters;
  prm.comm_warps = kWorkerWarps;
  prm.timeout_ns = problem.timeout_ns != 0 ? problem.timeout_ns : 10000000000ull;
  prm.act = static_cast<__nv_bfloat16 *>(act);
  prm.out = static_cast<__nv_bfloat16 *>(out);
  prm.x_work = static_cast<__nv_bfloat16 *>(x_work);
  prm.workspace = static_cast<char *>(workspace);
  prm.events = static_cast<std::uint32_t *>(events);
  if (team != nullptr) {
    prm.peers = team->peers;
  } else {
    prm.peers.n_pes = 1;
    prm.peers.my_pe = 0;
  }
  auto stream = static_cast<cudaStream_t>(driver.launch.stream);
  // The dependency counters start at zero in every launch; no peer reaches
  // this PE's counters before this launch has published its own partials.
  std::int64_t const counters =
      chain_counters_base(problem.layers, n_pes, pl.dn_tiles_n, pl.m_tiles);
  e = cudaMemsetAsync(static_cast<char *>(events) + kControlBytes + 4 * counters, 0,
                      4 * 2 * static_cast<std::int64_t>(problem.layers) * pl.m_tiles, stream);
  if (e != cudaSuccess) return cuda_fail(e, 11);
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  int const grid = problem.num_ctas > 0 ? problem.num_ctas : sms;
  e = pl.pairs ? launch_persistent<&mlp_chain_megakernel<true>, true,
                                   gemm_config<kChainBN, true>::smem_bytes>(device, grid, stream,
                                                                            maps, prm)
               : launch_persistent<&mlp_chain_megakernel<false>, false,
                                   gemm_config<kChainBN, false>::smem_bytes>(device, grid, stream,
                                                                             maps, prm);
  if (e != cudaSuccess) return cuda_fail(e, 14);
  return ok_status();
}

megacu_status check_chain(megacu_mlp_chain_problem const &p) {
  if (p.layers < 1 || p.layers > kMaxLayers) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "layers must be 1..64");
  }
  if (p.tokens <= 0 || p.hidden <= 0 || p.inter <= 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "invalid problem");
  }
  return ok_status();
}

}  // namespace

extern "C" megacu_status megacu_b200_swiglu_events_bytes(megacu_gemm_ar_problem_v2 problem,
                                                         std::int64_t *bytes) {
  if (bytes == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  swiglu_plan pl;
  megacu_status st = make_swiglu_plan(problem, pl);
  if (st.code == MEGACU_OK) *bytes = pl.events_bytes;
  return st;
}

extern "C" megacu_status megacu_cuda_gemm_swiglu_bf16(megacu_driver_view driver, void const *x,
                                                      void const *w_gate, void const *w_up,
                                                      void *act, void *events,
                                                      megacu_gemm_ar_problem_v2 problem) {
  return run_swiglu(driver, x, w_gate, w_up, act, events, problem);
}

extern "C" megacu_status megacu_b200_mlp_chain_sizes(megacu_mlp_chain_problem problem,
                                                     std::int32_t n_pes, std::int64_t sizes[5]) {
  if (sizes == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  megacu_status st = check_chain(problem);
  if (st.code != MEGACU_OK) return st;
  megacu_gemm_ar_problem_v2 const down = down_problem(problem);
  std::int64_t ws = 0, ev = 0, sev = 0;
  st = megacu_b200_workspace_bytes(down, n_pes, &ws);
  if (st.code == MEGACU_OK) st = megacu_b200_events_bytes(down, n_pes, &ev);
  if (st.code == MEGACU_OK) st = megacu_b200_swiglu_events_bytes(swiglu_problem(problem), &sev);
  if (st.code != MEGACU_OK) return st;
  // A single-launch chain uses workspace and events_down with its own layout.
  if (problem.single_launch) {
    chain_plan cp;
    st = make_chain_plan(problem, n_pes, cp);
    if (st.code != MEGACU_OK) return st;
    ws = ws > cp.workspace_bytes ? ws : cp.workspace_bytes;
    ev = ev > cp.events_bytes ? ev : cp.events_bytes;
  }
  sizes[0] = problem.tokens * problem.inter * 2;   // act, local
  sizes[1] = ws;                                   // down-projection workspace, symmetric
  sizes[2] = sev;                                  // SwiGLU events, local
  sizes[3] = ev;                                   // down-projection events, symmetric
  sizes[4] = problem.tokens * problem.hidden * 2;  // x_work, like out
  return ok_status();
}

extern "C" megacu_status megacu_cuda_mlp_chain_bf16(
    megacu_driver_view driver, void const *x, void const *const *w_gate,
    void const *const *w_up, void const *const *w_down, void *act, void *workspace,
    void *x_work, void *out, void *events_swiglu, void *events_down,
    megacu_mlp_chain_problem problem) {
  megacu_status st = check_chain(problem);
  if (st.code != MEGACU_OK) return st;
  if (w_gate == nullptr || w_up == nullptr || w_down == nullptr || x_work == nullptr ||
      out == nullptr) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  if (problem.single_launch) {
    return run_chain_single_launch(driver, x, w_gate, w_up, w_down, act, workspace, x_work, out,
                                   events_down, problem);
  }
  megacu_gemm_ar_problem_v2 const gu = swiglu_problem(problem);
  megacu_gemm_ar_problem_v2 const down = down_problem(problem);
  // Block l reads the previous block's output and writes out or x_work, so
  // that the last block writes out; consecutive blocks alternate.
  void const *in = x;
  for (std::int32_t l = 0; l < problem.layers; ++l) {
    void *dst = ((problem.layers - 1 - l) % 2 == 0) ? out : x_work;
    st = run_swiglu(driver, in, w_gate[l], w_up[l], act, events_swiglu, gu);
    if (st.code != MEGACU_OK) return st;
    st = megacu_cuda_gemm_allreduce_bf16(driver, act, w_down[l], workspace, dst, events_down, down);
    if (st.code != MEGACU_OK) return st;
    in = dst;
  }
  return ok_status();
}
