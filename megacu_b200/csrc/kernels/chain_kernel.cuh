// One persistent launch of a chain of tensor-parallel MLP blocks (benchmark
// config 5; no counterpart in megacu):
//
//   for l = 0 .. layers-1:   act     = silu(x_l @ gate_l) * (x_l @ up_l)    (local)
//                            x_{l+1} = sum over PEs of act @ down_l        (two-shot)
//
// The same warp roles, CTA pairs and pipelines as gemm_ar_megakernel, with
// 256 accumulator columns for both kinds of tile: a gate/up ("GU") tile holds
// 128 gate and the same 128 up columns and stores silu(g) * u into `act`; a
// down ("DN") tile holds 256 hidden columns and, on one PE, stores them as the
// block's output, on several PEs publishes them as this PE's partial for the
// tile's owner, whose workers reduce it and store the sum into every PE's
// copy of the block's output.
//
// Dependencies between blocks are carried by counters in the event tensor,
// one per (block, 128-row token block), all zeroed by the host before the
// launch:
//   act_ready[l][row]  +1 by each GU_l epilogue quarter of that row block
//                      (this PE); a DN_l tile waits for all of them;
//   x_ready[l][row]    +1 on every PE by the owner of each (DN_l tile,
//                      quarter) once its sum is stored there (one PE: by the
//                      DN_l epilogue quarter); a GU_{l+1} tile waits for all.
// A producer waits on its tile's counter before issuing its TMA loads. The
// GEMM queue hands out every GU_l and DN_l ticket before any of block l+1,
// and the exchange queue every sub-task of block l before any of block l+1,
// so every wait is for work already handed to a CTA that can finish it.
//
// Block outputs alternate between `out` and `x_work` so that the last lands
// in `out`. A single act buffer and a single plane of partial slots suffice:
// block l+1 writes a row block of either only after that row block of every
// PE's block l has been read.
//
// No loads here use cluster multicast.
#pragma once

#include "gemm_ar_kernel.cuh"

#if defined(__CUDACC__)
#define MEGACU_B200_CHAIN_HD __host__ __device__ __forceinline__
#else
#define MEGACU_B200_CHAIN_HD inline
#endif

namespace megacu_b200 {

inline constexpr int kChainMaxLayers = 6;
inline constexpr int kChainBN = 256;       // accumulator columns of every tile
inline constexpr int kChainActTile = 128;  // act columns of a GU tile
// Tensor maps: x, out, x_work, act, then gate, up and down of each block.
inline constexpr int kChainMapX = 0;
inline constexpr int kChainMapOut = 1;
inline constexpr int kChainMapWork = 2;
inline constexpr int kChainMapAct = 3;
inline constexpr int kChainMapLayer0 = 4;
inline constexpr int kChainMaps = kChainMapLayer0 + 3 * kChainMaxLayers;

struct chain_maps {
  CUtensorMap map[kChainMaps];
};

struct chain_params {
  std::int32_t tokens, hidden, inter, layers;
  std::int32_t m_tiles;     // 128-row token blocks
  std::int32_t gu_tiles_n;  // act column tiles (128 columns)
  std::int32_t dn_tiles_n;  // hidden column tiles (256 columns)
  std::int32_t gu_units, dn_units;  // GEMM tickets per block (pair tiles with CTA pairs)
  std::int32_t n_pes, my_pe, group_m;
  std::int32_t n_comm;      // exchange sub-tasks (owned DN tile x quarter) per block
  std::int32_t comm_warps;  // warps per CTA running them: the last comm_warps of 2..9
  std::int32_t reserved;
  std::uint64_t timeout_ns;  // bound of every cross-CTA and cross-GPU wait
  __nv_bfloat16 *act;        // [tokens, inter], this PE
  __nv_bfloat16 *out;        // [tokens, hidden], symmetric with several PEs
  __nv_bfloat16 *x_work;     // [tokens, hidden], symmetric with several PEs
  char *workspace;           // this PE's partial slots: DN tiles x 128 x 256 bf16
  std::uint32_t *events;     // control block + chain event words (symmetric)
  megacu::nvshmem::peer_table peers;
  unsigned long long *trace;
  std::int64_t trace_capacity;
};

// Event words after the control block: arrive[l][src][DN tile][quarter]
// (DN tile = row * dn_tiles_n + column, m_tiles * dn_tiles_n of them), then
// act_ready[l][row], then x_ready[l][row].
MEGACU_B200_CHAIN_HD std::int64_t chain_arrive_index(std::int32_t l, std::int32_t src,
                                                     std::int32_t tile, std::int32_t q,
                                                     std::int32_t n_pes, std::int32_t dn_tiles_n,
                                                     std::int32_t m_tiles) {
  std::int64_t const dn_tiles = static_cast<std::int64_t>(m_tiles) * dn_tiles_n;
  return ((static_cast<std::int64_t>(l) * n_pes + src) * dn_tiles + tile) * 4 + q;
}

MEGACU_B200_CHAIN_HD std::int64_t chain_counters_base(std::int32_t layers, std::int32_t n_pes,
                                                      std::int32_t dn_tiles_n,
                                                      std::int32_t m_tiles) {
  return static_cast<std::int64_t>(layers) * n_pes * m_tiles * dn_tiles_n * 4;
}

MEGACU_B200_CHAIN_HD std::int64_t chain_act_ready_index(std::int32_t l, std::int32_t row,
                                                        std::int32_t layers, std::int32_t n_pes,
                                                        std::int32_t dn_tiles_n,
                                                        std::int32_t m_tiles) {
  return chain_counters_base(layers, n_pes, dn_tiles_n, m_tiles) +
         static_cast<std::int64_t>(l) * m_tiles + row;
}

MEGACU_B200_CHAIN_HD std::int64_t chain_x_ready_index(std::int32_t l, std::int32_t row,
                                                      std::int32_t layers, std::int32_t n_pes,
                                                      std::int32_t dn_tiles_n,
                                                      std::int32_t m_tiles) {
  return chain_counters_base(layers, n_pes, dn_tiles_n, m_tiles) +
         static_cast<std::int64_t>(layers + l) * m_tiles + row;
}

MEGACU_B200_CHAIN_HD std::int64_t chain_events_bytes(std::int32_t layers, std::int32_t n_pes,
                                                     std::int32_t dn_tiles_n,
                                                     std::int32_t m_tiles) {
  return kControlBytes +
         4 * (chain_counters_base(layers, n_pes, dn_tiles_n, m_tiles) +
              2 * static_cast<std::int64_t>(layers) * m_tiles);
}

// 32-row quarters of token block `row` that hold tokens.
MEGACU_B200_CHAIN_HD std::int32_t chain_active_quarters(std::int32_t row, std::int32_t tokens) {
  std::int32_t const left = tokens - row * kBlockM;
  std::int32_t const q = (left + 31) / 32;
  return q < 4 ? q : 4;
}

namespace chain_detail {

__device__ __forceinline__ control_block *control(chain_params const &p) {
  return reinterpret_cast<control_block *>(p.events);
}

__device__ __forceinline__ void record_error(chain_params const &p, std::uint32_t code,
                                             std::uint32_t tile, std::uint32_t peer,
                                             std::uint32_t site) {
  control_block *c = control(p);
  if (atomicCAS(&c->error_code, 0u, code) == 0u) {
    c->error_info[0] = tile;
    c->error_info[1] = peer;
    c->error_info[2] = site;
  }
  atomicAdd(&c->counters[ctr_errors], 1ull);
}

__device__ __forceinline__ void count(chain_params const &p, int which, unsigned long long v) {
  atomicAdd(&control(p)->counters[which], v);
}

__device__ __forceinline__ void trace(chain_params const &p, std::uint32_t kind, std::uint32_t sub,
                                      std::uint32_t ticket, std::uint32_t tile,
                                      std::uint64_t t0) {
  if (p.trace == nullptr) return;
  std::uint32_t const i = atomicAdd(&control(p)->trace_count, 1u);
  if (static_cast<std::int64_t>(i) >= p.trace_capacity) return;
  unsigned long long *rec = p.trace + static_cast<std::int64_t>(i) * 4;
  rec[0] = static_cast<unsigned long long>(kind) | (static_cast<unsigned long long>(sub) << 8) |
           (static_cast<unsigned long long>(blockIdx.x) << 16) |
           (static_cast<unsigned long long>(ticket) << 32);
  rec[1] = tile;
  rec[2] = t0;
  rec[3] = ptx::now_ns();
}

// Waits until the counter reaches `target` (it only grows during a launch).
// Bounded: gives up on the abort word or after `timeout_ns`.
__device__ __forceinline__ bool wait_count(std::uint32_t const *counter, std::uint32_t target,
                                           std::uint32_t const *abort_word,
                                           std::uint64_t timeout_ns) {
  if (ptx::ld_acquire_sys(counter) >= target) return true;
  std::uint64_t const start = ptx::now_ns();
  for (std::uint32_t spin = 1;; ++spin) {
    __nanosleep(spin < 64 ? 64 : 256);
    if (ptx::ld_relaxed_sys(counter) >= target && ptx::ld_acquire_sys(counter) >= target) {
      return true;
    }
    if ((spin & 15u) == 0) {
      if (ptx::ld_relaxed_gpu(abort_word) != 0) return false;
      if (ptx::now_ns() - start > timeout_ns) return false;
    }
  }
}

// A GEMM ticket: block, kind (0 = GU, 1 = DN) and the ticket within the job.
struct chain_job {
  std::int32_t layer;
  std::int32_t kind;
  std::int32_t unit;
};

__device__ __forceinline__ chain_job decode(chain_params const &p, std::int32_t ticket) {
  std::int32_t const per_layer = p.gu_units + p.dn_units;
  chain_job j;
  j.layer = ticket / per_layer;
  std::int32_t const w = ticket % per_layer;
  j.kind = w < p.gu_units ? 0 : 1;
  j.unit = j.kind == 0 ? w : w - p.gu_units;
  return j;
}

// Output buffer of block l: the blocks alternate so the last writes out.
__device__ __forceinline__ __nv_bfloat16 *block_out(chain_params const &p, std::int32_t l) {
  return ((p.layers - 1 - l) % 2 == 0) ? p.out : p.x_work;
}

__device__ __forceinline__ int block_out_map(chain_params const &p, std::int32_t l) {
  return ((p.layers - 1 - l) % 2 == 0) ? kChainMapOut : kChainMapWork;
}

// Exchange worker (several PEs): sub-tasks (block, owned DN tile, quarter) in
// order; for each: acquire every PE's partial of the quarter, then for each
// 64-column block load it from every PE's slot, sum in PE order in fp32,
// round to bf16, transpose 32 x 64 through `xpose` and store the rows into
// every PE's copy of the block's output; finally fence at system scope and
// add one to x_ready[block][row] on every PE.
__device__ __forceinline__ void exchange(chain_params const &p, tile_schedule const &sched_dn,
                                         std::uint32_t epoch, std::uint32_t *my_events,
                                         std::uint32_t const *abort_word, std::uint8_t *xpose,
                                         std::uint32_t lane) {
  constexpr int kBlocks = kChainBN / 64;
  constexpr std::int64_t kSlotBytes = std::int64_t(kBlockM) * kChainBN * 2;
  constexpr std::int64_t kVecStride = kBlockM * 16;
  control_block *ctrl = control(p);
  std::int32_t const total = p.layers * p.n_comm;
  for (;;) {
    std::uint32_t const ticket = detail::draw_ticket(&ctrl->reduce_ticket, lane);
    if (ticket >= static_cast<std::uint32_t>(total)) break;
    std::int32_t const layer = static_cast<std::int32_t>(ticket) / p.n_comm;
    std::int32_t const rem = static_cast<std::int32_t>(ticket) % p.n_comm;
    std::int32_t const quarter = rem % 4;
    std::int32_t const r = (rem / 4) * p.n_pes + p.my_pe;  // two-shot: owned tiles
    tile_coord const c = locate(sched_dn, r);
    std::int32_t const tile = c.tile_row * p.dn_tiles_n + c.tile_col;
    std::int32_t const row0 = c.tile_row * kBlockM + quarter * 32;
    if (row0 >= p.tokens) continue;  // a quarter without tokens: nothing to reduce or count
    if constexpr (kCheckBounds) {
      std::int64_t const dn_tiles = static_cast<std::int64_t>(p.m_tiles) * p.dn_tiles_n;
      std::int64_t const words =
          (chain_events_bytes(p.layers, p.n_pes, p.dn_tiles_n, p.m_tiles) - kControlBytes) / 4;
      bool const in =
          layer < p.layers && tile >= 0 && tile < dn_tiles && c.owner == p.my_pe &&
          chain_arrive_index(layer, p.n_pes - 1, tile, 3, p.n_pes, p.dn_tiles_n, p.m_tiles) <
              chain_counters_base(p.layers, p.n_pes, p.dn_tiles_n, p.m_tiles) &&
          chain_x_ready_index(layer, c.tile_row, p.layers, p.n_pes, p.dn_tiles_n, p.m_tiles) <
              words;
      if (!in) {
        if (lane == 0) record_error(p, err_bounds, ticket, static_cast<std::uint32_t>(tile), 32);
        continue;  // nothing reduced or counted: the waiting PEs time out
      }
    }

    bool ok = true;
    if (static_cast<std::int32_t>(lane) < p.n_pes) {
      ok = detail::wait_flag(
          my_events + chain_arrive_index(layer, lane, tile, quarter, p.n_pes, p.dn_tiles_n,
                                         p.m_tiles),
          epoch, abort_word, p.timeout_ns);
      if (!ok) record_error(p, err_remote_timeout, tile, lane, 18);
    }
    if (!__all_sync(0xffffffffu, ok)) break;
    __syncwarp();
    std::uint64_t const t0 = ptx::now_ns();
    __nv_bfloat16 *const dst_local = block_out(p, layer);
    std::int64_t const in_quarter = detail::slot_offset(0, tile, p.dn_tiles_n * p.m_tiles, kSlotBytes) +
                                    (static_cast<std::int64_t>(quarter) * 32 + lane) * 16;
#pragma unroll 1
    for (int cb = 0; cb < kBlocks; ++cb) {
      if (c.tile_col * kChainBN + cb * 64 >= p.hidden) break;
      float acc[8][8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = 0.0f;
      }
#pragma unroll 1
      for (std::int32_t src = 0; src < p.n_pes; src += 2) {
        bool const pair = src + 1 < p.n_pes;
        char const *base0 = p.peers.translate(p.workspace, src) + in_quarter;
        uint4 w0[8], w1[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) w0[g] = ptx::ld_cg_v4(base0 + (cb * 8 + g) * kVecStride);
        if (pair) {
          char const *base1 = p.peers.translate(p.workspace, src + 1) + in_quarter;
#pragma unroll
          for (int g = 0; g < 8; ++g) w1[g] = ptx::ld_cg_v4(base1 + (cb * 8 + g) * kVecStride);
        }
#pragma unroll
        for (int g = 0; g < 8; ++g) detail::add_bf16x8(acc[g], w0[g]);
        if (pair) {
#pragma unroll
          for (int g = 0; g < 8; ++g) detail::add_bf16x8(acc[g], w1[g]);
        }
      }
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        uint4 q;
        q.x = ptx::pack_bf16x2(acc[g][0], acc[g][1]);
        q.y = ptx::pack_bf16x2(acc[g][2], acc[g][3]);
        q.z = ptx::pack_bf16x2(acc[g][4], acc[g][5]);
        q.w = ptx::pack_bf16x2(acc[g][6], acc[g][7]);
        *reinterpret_cast<uint4 *>(xpose + lane * 128 + ((g ^ (lane & 7)) * 16)) = q;
      }
      __syncwarp();
      std::int32_t const gg = lane % 8;
      std::int32_t const col = c.tile_col * kChainBN + cb * 64 + gg * 8;
      for (std::int32_t d = 0; d < p.n_pes; ++d) {
        std::int32_t const pe = (p.my_pe + 1 + d) % p.n_pes;
        __nv_bfloat16 *dst = p.peers.translate(dst_local, pe);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          std::int32_t const rr = i * 4 + static_cast<std::int32_t>(lane) / 8;
          uint4 const q =
              *reinterpret_cast<uint4 const *>(xpose + rr * 128 + ((gg ^ (rr & 7)) * 16));
          if (row0 + rr < p.tokens && col < p.hidden) {
            ptx::st_v4(dst + static_cast<std::int64_t>(row0 + rr) * p.hidden + col, q);
          }
        }
      }
      __syncwarp();
    }
    // The quarter's rows are stored on every PE: publish them.
    ptx::fence_acq_rel_sys();
    __syncwarp();
    if (static_cast<std::int32_t>(lane) < p.n_pes) {
      std::uint32_t *theirs = p.peers.translate(my_events, lane);
      ptx::red_release_sys_add(
          theirs + chain_x_ready_index(layer, c.tile_row, p.layers, p.n_pes, p.dn_tiles_n,
                                       p.m_tiles),
          1u);
    }
    __syncwarp();
    if (lane == 0) {
      count(p, ctr_reduce_tasks, 1);
      count(p, ctr_partial_acquire, p.n_pes);
      count(p, ctr_final_publish, p.n_pes);
      trace(p, 2, (layer << 4) | quarter, ticket, tile, t0);
    }
  }
}

}  // namespace chain_detail

template <bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    mlp_chain_megakernel(const __grid_constant__ chain_maps maps,
                         const __grid_constant__ chain_params p) {
  using cfg = gemm_config<kChainBN, kPair>;
  constexpr int BN = kChainBN;
  constexpr std::int64_t kSlotBytes = std::int64_t(kBlockM) * BN * 2;

  extern __shared__ std::uint8_t smem_raw[];
  std::uint32_t const raw_addr = ptx::smem_addr(smem_raw);
  std::uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  std::uint8_t *stages = smem;
  std::uint8_t *reduce_smem = smem + cfg::stages * cfg::stage_bytes;
  auto *bars = reinterpret_cast<std::uint64_t *>(reduce_smem + cfg::reduce_bytes);
  std::uint64_t *full = bars;
  std::uint64_t *empty = full + cfg::stages;
  std::uint64_t *acc_full = empty + cfg::stages;
  std::uint64_t *acc_empty = acc_full + 2;
  std::uint64_t *task_full = acc_empty + 2;
  std::uint64_t *task_empty = task_full + kTaskRing;
  std::uint64_t *mma_done = task_empty + kTaskRing;
  auto *ring = reinterpret_cast<std::int32_t volatile *>(mma_done + 1);
  auto *tmem_slot = reinterpret_cast<std::uint32_t *>(const_cast<std::int32_t *>(ring) + kTaskRing);
  auto *epoch_slot = tmem_slot + 1;

  int const warp = threadIdx.x / 32;
  std::uint32_t const lane = threadIdx.x % 32;
  control_block *ctrl = chain_detail::control(p);
  std::uint32_t const *abort_word = &ctrl->error_code;
  tile_schedule const sched_gu{p.m_tiles, p.gu_tiles_n, 1, mode_allreduce, p.group_m};
  tile_schedule const sched_dn{p.m_tiles, p.dn_tiles_n, p.n_pes, mode_allreduce, p.group_m};
  std::int32_t const total_units = p.layers * (p.gu_units + p.dn_units);
  std::uint32_t const cta_rank = kPair ? ptx::cluster_ctarank() : 0u;
  bool const leader = cta_rank == 0;
  // Raster index (within its job) of the tile this CTA computes for a ticket.
  auto tile_of = [&](chain_detail::chain_job const &j) {
    tile_schedule const &s = j.kind == 0 ? sched_gu : sched_dn;
    return kPair ? pair_raster(s, j.unit, static_cast<std::int32_t>(cta_rank)) : j.unit;
  };
  auto k_blocks_of = [&](chain_detail::chain_job const &j) {
    return ((j.kind == 0 ? p.hidden : p.inter) + kBlockK - 1) / kBlockK;
  };
  // Pipeline waits: a stage or accumulator may wait on another GPU here (a
  // producer's dependency), so they get the cross-GPU bound as well.
  std::uint64_t const pipe_timeout = p.timeout_ns + kLocalTimeoutNs;
  auto pipe_wait = [&](std::uint64_t *bar, std::uint32_t parity) {
    return kPair ? ptx::mbar_wait_cluster(bar, parity, abort_word, pipe_timeout)
                 : ptx::mbar_wait(bar, parity, abort_word, pipe_timeout);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < cfg::stages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&acc_full[b], 1);
      ptx::mbar_init(&acc_empty[b], kPair ? 8 : 4);
    }
    for (int i = 0; i < kTaskRing; ++i) {
      ptx::mbar_init(&task_full[i], 1);
      ptx::mbar_init(&task_empty[i], kPair ? 10 : 5);
    }
    ptx::mbar_init(mma_done, 1);
    ptx::fence_barrier_init();
    *epoch_slot = ptx::ld_relaxed_gpu(&ctrl->launch_count) + 1u;
    for (int i = 0; i < kChainMapLayer0 + 3 * p.layers; ++i) {
      ptx::prefetch_tensor_map(&maps.map[i]);
    }
  }
  if (warp == 1) {
    if constexpr (kPair) {
      ptx::tmem_alloc_pair(tmem_slot, cfg::tmem_columns);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(tmem_slot, cfg::tmem_columns);
      ptx::tmem_relinquish();
    }
  }
  ptx::tc_fence_before_sync();
  __syncthreads();
  if constexpr (kPair) {
    ptx::cluster_sync();
  }
  ptx::tc_fence_after_sync();
  std::uint32_t const tmem_base = *tmem_slot;
  std::uint32_t const epoch = *epoch_slot;
  std::uint32_t *const my_events = detail::event_words(p.events);

  if (warp == 0) {
    // ---------------- task fetcher + TMA producer ----------------
    if (lane == 0) {
      std::uint32_t it = 0;
      bool ok = true;
      for (std::uint32_t n = 0; ok; ++n) {
        std::uint32_t const slot = n % kTaskRing;
        std::int32_t t = -1;
        if (leader) {
          if (!pipe_wait(&task_empty[slot], ((n / kTaskRing) & 1u) ^ 1u)) {
            chain_detail::record_error(p, err_local_timeout, 0, 0, 11);
            break;
          }
          std::uint32_t const ticket = atomicAdd(&ctrl->gemm_ticket, 1u);
          t = ticket < static_cast<std::uint32_t>(total_units) ? static_cast<std::int32_t>(ticket)
                                                               : -1;
          ring[slot] = t;
          if constexpr (kPair) {
            ptx::st_shared_remote(ptx::map_to_rank(const_cast<std::int32_t *>(&ring[slot]), 1), t);
            ptx::mbar_arrive_remote(ptx::map_to_rank(&task_full[slot], 1));
          }
          ptx::mbar_arrive(&task_full[slot]);
        } else {
          if (!pipe_wait(&task_full[slot], (n / kTaskRing) & 1u)) {
            chain_detail::record_error(p, err_local_timeout, 0, 1, 11);
            break;
          }
          t = ring[slot];
          ptx::mbar_arrive_remote(ptx::map_to_rank(&task_empty[slot], 0));
        }
        if (t < 0) break;
        chain_detail::chain_job const j = chain_detail::decode(p, t);
        std::int32_t const r = tile_of(j);
        tile_coord const c = locate(j.kind == 0 ? sched_gu : sched_dn, r);
        // The tile's input rows: block l's output for GU_{l+1}, act for DN_l.
        std::uint32_t const *dep = nullptr;
        std::uint32_t target = 0;
        std::int32_t const aq = chain_active_quarters(c.tile_row, p.tokens);
        if (j.kind == 0 && j.layer > 0) {
          dep = my_events + chain_x_ready_index(j.layer - 1, c.tile_row, p.layers, p.n_pes,
                                                p.dn_tiles_n, p.m_tiles);
          target = static_cast<std::uint32_t>(aq * p.dn_tiles_n);
        } else if (j.kind == 1) {
          dep = my_events + chain_act_ready_index(j.layer, c.tile_row, p.layers, p.n_pes,
                                                  p.dn_tiles_n, p.m_tiles);
          target = static_cast<std::uint32_t>(aq * p.gu_tiles_n);
        }
        if constexpr (kCheckBounds) {
          if (j.layer >= p.layers || c.tile_row < 0 || c.tile_row >= p.m_tiles) {
            chain_detail::record_error(p, err_bounds, static_cast<std::uint32_t>(t), cta_rank, 35);
            break;
          }
        }
        if (dep != nullptr) {
          if (!chain_detail::wait_count(dep, target, abort_word, p.timeout_ns)) {
            chain_detail::record_error(p, err_remote_timeout, static_cast<std::uint32_t>(t),
                                       cta_rank, 12);
            break;
          }
          ptx::fence_proxy_async_global();  // TMA reads what the acquire made visible
        }
        CUtensorMap const *map_a;
        CUtensorMap const *map_b;
        CUtensorMap const *map_b2;
        if (j.kind == 0) {
          map_a = &maps.map[j.layer == 0 ? kChainMapX : chain_detail::block_out_map(p, j.layer - 1)];
          map_b = &maps.map[kChainMapLayer0 + 3 * j.layer + 0];
          map_b2 = &maps.map[kChainMapLayer0 + 3 * j.layer + 1];
        } else {
          map_a = &maps.map[kChainMapAct];
          map_b = &maps.map[kChainMapLayer0 + 3 * j.layer + 2];
          map_b2 = map_b;
        }
        // GU: gate and up columns [tile_col * 128, + 128) (a pair's leader
        // stages gate, its follower up); DN: hidden columns [tile_col * 256,
        // + 256), split between the CTAs of a pair.
        std::int32_t const b_col0 =
            j.kind == 0 ? c.tile_col * kChainActTile
                        : c.tile_col * BN + static_cast<std::int32_t>(cta_rank) * cfg::b_cols;
        CUtensorMap const *pair_b = (j.kind == 0 && cta_rank == 1) ? map_b2 : map_b;
        std::int32_t const k_blocks = k_blocks_of(j);
        for (std::int32_t kb = 0; kb < k_blocks; ++kb, ++it) {
          std::uint32_t const s = it % cfg::stages;
          if (!pipe_wait(&empty[s], ((it / cfg::stages) & 1u) ^ 1u)) {
            chain_detail::record_error(p, err_local_timeout, static_cast<std::uint32_t>(t), 0, 13);
            ok = false;
            break;
          }
          std::uint8_t *sa = stages + s * cfg::stage_bytes;
          std::uint8_t *sb = sa + cfg::a_bytes;
          if constexpr (kPair) {
            if (leader && it >= static_cast<std::uint32_t>(cfg::stages)) {
              ptx::mbar_arrive_remote_relaxed(ptx::map_to_rank(&empty[s], 1));
            }
            std::uint32_t const bar = ptx::map_to_rank(&full[s], 0);
            if (leader) ptx::mbar_arrive_expect_tx(&full[s], cfg::tx_bytes);
            ptx::tma_load_2d_pair(map_a, bar, sa, kb * kBlockK, c.tile_row * kBlockM);
#pragma unroll
            for (int panel = 0; panel < cfg::b_cols / 64; ++panel) {
              ptx::tma_load_2d_pair(pair_b, bar, sb + panel * cfg::b_panel_bytes,
                                    b_col0 + panel * 64, kb * kBlockK);
            }
          } else {
            ptx::mbar_arrive_expect_tx(&full[s], cfg::tx_bytes);
            ptx::tma_load_2d(map_a, &full[s], sa, kb * kBlockK, c.tile_row * kBlockM);
#pragma unroll
            for (int panel = 0; panel < BN / 64; ++panel) {
              CUtensorMap const *map = (j.kind == 0 && panel >= 2) ? map_b2 : map_b;
              std::int32_t const col = j.kind == 0 ? b_col0 + (panel % 2) * 64 : b_col0 + panel * 64;
              ptx::tma_load_2d(map, &full[s], sb + panel * cfg::b_panel_bytes, col, kb * kBlockK);
            }
          }
        }
      }
      for (std::uint32_t back = 1; leader && back <= cfg::stages && back <= it; ++back) {
        std::uint32_t const i = it - back;
        kPair ? ptx::mbar_wait_cluster(&full[i % cfg::stages], (i / cfg::stages) & 1u, nullptr,
                                       pipe_timeout)
              : ptx::mbar_wait(&full[i % cfg::stages], (i / cfg::stages) & 1u, nullptr,
                               pipe_timeout);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- tcgen05.mma issuer ----------------
    if (lane == 0 && leader) {
      std::uint32_t const idesc = ptx::idesc_bf16_f32(kPair ? 2 * kBlockM : kBlockM, BN, true);
      std::uint32_t it = 0;
      for (std::uint32_t n = 0;; ++n) {
        std::uint32_t const slot = n % kTaskRing;
        if (!ptx::mbar_wait(&task_full[slot], (n / kTaskRing) & 1u, abort_word, pipe_timeout)) {
          chain_detail::record_error(p, err_local_timeout, 0, 0, 14);
          break;
        }
        std::int32_t const t = ring[slot];
        ptx::mbar_arrive(&task_empty[slot]);
        if (t < 0) break;
        std::int32_t const k_blocks = k_blocks_of(chain_detail::decode(p, t));
        std::uint32_t const buf = n & 1u;
        if (!pipe_wait(&acc_empty[buf], ((n >> 1) & 1u) ^ 1u)) {
          chain_detail::record_error(p, err_local_timeout, static_cast<std::uint32_t>(t), 0, 15);
          break;
        }
        ptx::tc_fence_after_sync();
        std::uint32_t const d_tmem = tmem_base + buf * BN;
        bool ok = true;
        for (std::int32_t kb = 0; kb < k_blocks; ++kb, ++it) {
          std::uint32_t const s = it % cfg::stages;
          if (!pipe_wait(&full[s], (it / cfg::stages) & 1u)) {
            chain_detail::record_error(p, err_local_timeout, static_cast<std::uint32_t>(t), 0, 16);
            ok = false;
            break;
          }
          ptx::tc_fence_after_sync();
          std::uint32_t const a_addr = ptx::smem_addr(stages + s * cfg::stage_bytes);
          std::uint32_t const b_addr = a_addr + cfg::a_bytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            std::uint64_t const a_desc = ptx::smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            std::uint64_t const b_desc =
                ptx::smem_desc_sw128(b_addr + kk * 2048, cfg::b_panel_bytes, 1024);
            std::uint32_t const acc = (kb > 0 || kk > 0) ? 1u : 0u;
            if constexpr (kPair) {
              ptx::umma_f16_pair(d_tmem, a_desc, b_desc, idesc, acc);
            } else {
              ptx::umma_f16(d_tmem, a_desc, b_desc, idesc, acc);
            }
          }
          if constexpr (kPair) {
            ptx::umma_commit_pair(&empty[s]);
          } else {
            ptx::umma_commit(&empty[s]);
          }
        }
        if (!ok) break;
        if constexpr (kPair) {
          ptx::umma_commit_pair(&acc_full[buf]);
        } else {
          ptx::umma_commit(&acc_full[buf]);
        }
      }
      if constexpr (kPair) {
        ptx::umma_commit_pair(mma_done);
      } else {
        ptx::umma_commit(mma_done);
      }
      ptx::mbar_wait(mma_done, 0, nullptr, pipe_timeout);
    }
    __syncwarp();
  } else if (warp < kReduceWarp0) {
    // ---------------- epilogue ----------------
    std::int32_t const quarter = warp % 4;
    std::int32_t const row_in_tile = quarter * 32 + static_cast<std::int32_t>(lane);
    for (std::uint32_t n = 0;; ++n) {
      std::uint32_t const slot = n % kTaskRing;
      if (!__all_sync(0xffffffffu,
                      pipe_wait(&task_full[slot], (n / kTaskRing) & 1u))) {
        if (lane == 0) chain_detail::record_error(p, err_local_timeout, 0, cta_rank, 17);
        break;
      }
      std::int32_t const t = __shfl_sync(0xffffffffu, ring[slot], 0);
      if (lane == 0) {
        if (leader) {
          ptx::mbar_arrive(&task_empty[slot]);
        } else {
          ptx::mbar_arrive_remote(ptx::map_to_rank(&task_empty[slot], 0));
        }
      }
      if (t < 0) break;
      chain_detail::chain_job const j = chain_detail::decode(p, t);
      std::int32_t const r = tile_of(j);
      std::uint32_t const buf = n & 1u;
      if (!__all_sync(0xffffffffu, pipe_wait(&acc_full[buf], (n >> 1) & 1u))) {
        if (lane == 0) {
          chain_detail::record_error(p, err_local_timeout, static_cast<std::uint32_t>(t),
                                     cta_rank, 19);
        }
        break;
      }
      if constexpr (kPair) {
        if (leader && warp == kEpilogueWarp0 && lane == 0) {
          ptx::mbar_arrive_remote(ptx::map_to_rank(&acc_full[buf], 1));
        }
      }
      ptx::tc_fence_after_sync();
      std::uint64_t const t0 = ptx::now_ns();
      tile_coord const c = locate(j.kind == 0 ? sched_gu : sched_dn, r);
      std::int32_t const grow = c.tile_row * kBlockM + row_in_tile;
      std::uint32_t const t_row = tmem_base + (static_cast<std::uint32_t>(quarter * 32) << 16) +
                                  buf * BN;
      bool const active = c.tile_row * kBlockM + quarter * 32 < p.tokens;
      std::int32_t const dn_tile = c.tile_row * p.dn_tiles_n + c.tile_col;

      if (j.kind == 0) {
        // act[row, col] = silu(gate) * up (accumulator columns col, 128 + col).
        std::int32_t const acol0 = c.tile_col * kChainActTile;
#pragma unroll 1
        for (int ch = 0; active && ch < BN / 64; ++ch) {
          std::uint32_t g[32], u[32];
          ptx::tmem_load_32x32b_x32(t_row + ch * 32, g);
          ptx::tmem_load_32x32b_x32(t_row + BN / 2 + ch * 32, u);
          ptx::tmem_wait_load();
          if (grow < p.tokens) {
            __nv_bfloat16 *dst = p.act + static_cast<std::int64_t>(grow) * p.inter;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              std::int32_t const col = acol0 + ch * 32 + jj * 8;
              if (col < p.inter) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  float const x = __uint_as_float(g[8 * jj + e]);
                  f[e] = x / (1.0f + __expf(-x)) * __uint_as_float(u[8 * jj + e]);
                }
                uint4 q;
                q.x = ptx::pack_bf16x2(f[0], f[1]);
                q.y = ptx::pack_bf16x2(f[2], f[3]);
                q.z = ptx::pack_bf16x2(f[4], f[5]);
                q.w = ptx::pack_bf16x2(f[6], f[7]);
                ptx::st_v4(dst + col, q);
              }
            }
          }
        }
      } else {
        __nv_bfloat16 *const xout = chain_detail::block_out(p, j.layer);
        char *const slot_base =
            p.workspace + detail::slot_offset(0, dn_tile, p.dn_tiles_n * p.m_tiles, kSlotBytes);
#pragma unroll 1
        for (int ch = 0; active && ch < BN / 32; ++ch) {
          std::uint32_t v[32];
          ptx::tmem_load_32x32b_x32(t_row + ch * 32, v);
          ptx::tmem_wait_load();
          if (p.n_pes == 1) {
            // One PE: the block's output row, as written.
            if (grow < p.tokens) {
              __nv_bfloat16 *dst = xout + static_cast<std::int64_t>(grow) * p.hidden;
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                std::int32_t const col = c.tile_col * BN + ch * 32 + jj * 8;
                if (col < p.hidden) {
                  uint4 q;
                  q.x = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 0]), __uint_as_float(v[8 * jj + 1]));
                  q.y = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 2]), __uint_as_float(v[8 * jj + 3]));
                  q.z = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 4]), __uint_as_float(v[8 * jj + 5]));
                  q.w = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 6]), __uint_as_float(v[8 * jj + 7]));
                  ptx::st_v4(dst + col, q);
                }
              }
            }
          } else {
            // This PE's partial (bf16 wire) in its own slot.
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              uint4 q;
              q.x = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 0]), __uint_as_float(v[8 * jj + 1]));
              q.y = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 2]), __uint_as_float(v[8 * jj + 3]));
              q.z = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 4]), __uint_as_float(v[8 * jj + 5]));
              q.w = ptx::pack_bf16x2(__uint_as_float(v[8 * jj + 6]), __uint_as_float(v[8 * jj + 7]));
              std::int64_t const vec = ch * 4 + jj;
              ptx::st_v4(slot_base + (vec * kBlockM + row_in_tile) * 16, q);
            }
          }
        }
      }
      ptx::tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (leader) {
          ptx::mbar_arrive(&acc_empty[buf]);
        } else {
          ptx::mbar_arrive_remote(ptx::map_to_rank(&acc_empty[buf], 0));
        }
      }
      if (lane == 0 && quarter == 0) {
        chain_detail::count(p, ctr_gemm_tasks, 1);
        chain_detail::trace(p, 0, static_cast<std::uint32_t>((j.layer << 1) | j.kind),
                            static_cast<std::uint32_t>(t), static_cast<std::uint32_t>(dn_tile), t0);
      }
      if (!active) continue;
      // Publish the quarter: the data is in this PE's memory, so a GPU-scope
      // fence covers it (its readers acquire the counter or flag).
      ptx::fence_acq_rel_gpu();
      __syncwarp();
      if constexpr (kCheckBounds) {
        bool const in = j.layer < p.layers && c.tile_row < p.m_tiles &&
                        (j.kind == 0 || (dn_tile < p.m_tiles * p.dn_tiles_n && c.owner >= 0 &&
                                         c.owner < p.n_pes));
        if (!in) {
          if (lane == 0) {
            chain_detail::record_error(p, err_bounds, static_cast<std::uint32_t>(t),
                                       static_cast<std::uint32_t>(dn_tile), 34);
          }
          continue;  // not published: its consumers time out
        }
      }
      if (lane == 0) {
        if (j.kind == 0) {
          atomicAdd(my_events + chain_act_ready_index(j.layer, c.tile_row, p.layers, p.n_pes,
                                                      p.dn_tiles_n, p.m_tiles),
                    1u);
        } else if (p.n_pes == 1) {
          atomicAdd(my_events + chain_x_ready_index(j.layer, c.tile_row, p.layers, p.n_pes,
                                                    p.dn_tiles_n, p.m_tiles),
                    1u);
        } else {
          std::uint32_t *flags = p.peers.translate(my_events, c.owner);
          ptx::publish_local_data(flags + chain_arrive_index(j.layer, p.my_pe, dn_tile, quarter,
                                                             p.n_pes, p.dn_tiles_n, p.m_tiles),
                                  epoch);
        }
        chain_detail::count(p, ctr_partial_publish, 1);
      }
    }
  }

  // ---------------- exchange workers (several PEs) ----------------
  int const first_comm_warp = kThreads / 32 - p.comm_warps;
  if (p.n_pes > 1 && warp >= first_comm_warp) {
    int const worker = warp - kEpilogueWarp0;
    std::uint8_t *xpose = reduce_smem + worker * (32 * 128);
    chain_detail::exchange(p, sched_dn, epoch, my_events, abort_word, xpose, lane);
    if (blockIdx.x == 0 && warp == first_comm_warp) {
      // The last block's output on this PE is complete once every owner has
      // counted each of its row blocks.
      bool ok = true;
      for (std::int32_t row = static_cast<std::int32_t>(lane); row < p.m_tiles; row += 32) {
        std::uint32_t const target =
            static_cast<std::uint32_t>(chain_active_quarters(row, p.tokens) * p.dn_tiles_n);
        std::uint32_t const *counter =
            my_events + chain_x_ready_index(p.layers - 1, row, p.layers, p.n_pes, p.dn_tiles_n,
                                            p.m_tiles);
        if (!chain_detail::wait_count(counter, target, abort_word, p.timeout_ns)) {
          chain_detail::record_error(p, err_remote_timeout, static_cast<std::uint32_t>(row), 0, 20);
          ok = false;
          break;
        }
      }
      if (__all_sync(0xffffffffu, ok) && lane == 0) {
        chain_detail::count(p, ctr_final_acquire, p.n_pes);
      }
    }
  }

  // ---------------- teardown ----------------
  __syncwarp();
  ptx::tc_fence_before_sync();
  __syncthreads();
  if constexpr (kPair) {
    ptx::cluster_sync();
  }
  ptx::tc_fence_after_sync();
  if (warp == 1) {
    if constexpr (kPair) {
      ptx::tmem_dealloc_pair(tmem_base, cfg::tmem_columns);
    } else {
      ptx::tmem_dealloc(tmem_base, cfg::tmem_columns);
    }
  }
  if (threadIdx.x == 0) {
    __threadfence();
    std::uint32_t const done = atomicAdd(&ctrl->done_ctas, 1u);
    if (done == gridDim.x - 1) {
      __threadfence();
      ctrl->gemm_ticket = 0;
      ctrl->reduce_ticket = 0;
      ctrl->workers_done = 0;
      ctrl->trace_count = 0;
      ctrl->launch_count = epoch;
      atomicAdd(&ctrl->counters[ctr_launches], 1ull);
      __threadfence();
      atomicExch(&ctrl->done_ctas, 0u);
    }
  }
}

}  // namespace megacu_b200

#undef MEGACU_B200_CHAIN_HD
