// Tensor-parallel MLP blocks (no counterpart in megacu):
//   act   = silu(x @ w_gate) * (x @ w_up)      column-parallel, local
//   x_out = allreduce_pe(act @ w_down)          row-parallel, fused exchange
// megacu_cuda_gemm_swiglu_bf16 is the first line as one persistent launch of
// the megakernel's SwiGLU variant; megacu_cuda_mlp_chain_bf16 runs `layers`
// such blocks back to back, each one SwiGLU launch and one fused GEMM +
// allreduce launch (megacu_cuda_gemm_allreduce_bf16), the output of one block
// feeding the next.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include <megacu_b200.h>

#include "kernels/gemm_ar_kernel.cuh"
#include "kernels/launch.cuh"
#include "tma_map.h"

namespace {

using namespace megacu_b200;

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
