// Persistent sm_100a megakernel: tensor-parallel bf16 GEMM tiles (fp32
// accumulate in TMEM) fused with the allreduce / reduce-scatter of their
// outputs over NVLink peer memory.
//
// This is megacu's phased GEMM+AllReduce (megacu_gemm_allreduce_phased.cu:
// 56-148, three tasks per tile: 0 = GEMM tile producer, 1 = sync,
// 2 = allreduce consumer, with an event tensor between task 0 and task 2)
// re-designed for B200:
//
//  * one CTA per SM, 10 warps with fixed roles
//      warp 0      task fetcher + TMA producer (GEMM task queue)
//      warp 1      TMEM allocator + tcgen05.mma issuer (one thread)
//      warps 2..5  epilogue: TMEM -> registers -> bf16/fp32 -> this PE's own
//                  partial slot, then publish (task 0's "after" hook); once
//                  the GEMM queue is drained they join the workers below
//      warps 6..9  workers: one raster-ordered queue of task-2 sub-tasks
//                  (acquire, PE-order fp32 sum of every PE's partial read
//                  over NVLink, store into this PE's out, or into every PE's
//                  out in two-shot allreduce)
//    optionally as 2-CTA clusters whose pair computes 256-row tiles with
//    cta_group::2 MMAs (kPair below);
//  * the static tile_grid dispatcher (tile = blockIdx + i * gridDim,
//    tile_grid_device.cuh:13-23) is replaced by device task queues: an
//    atomic ticket per queue, tickets mapped to tiles by tile_schedule.h;
//  * the event tensor holds one arrive flag per (PE, tile, 32-row quarter)
//    and, for two-shot allreduce, one done flag per PE, tagged with the
//    call's epoch, stored after a fence and acquired with ld.acquire.sys
//    under a bounded wait;
//  * every partial crosses NVLink as a load by its consumer: producers write
//    only their own memory (so a GPU-scope fence covers them) and send 4-byte
//    flags;
//  * the all-gather variant (kGather) turns the exchange around: the workers
//    copy the other PEs' A shards over NVLink into a local gathered A while
//    the GEMM computes the tiles whose rows are already here, each tile
//    waiting on a counter of its tile row's copied chunks.
//
// No loads here use cluster multicast.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include <megacu/backends/nvshmem.h>

#include "layout.h"
#include "sm100_ptx.cuh"
#include "tile_schedule.h"

namespace megacu_b200 {

inline constexpr int kBlockM = 128;
inline constexpr int kBlockK = 64;
inline constexpr int kThreads = 320;
inline constexpr int kTaskRing = 4;
inline constexpr int kEpilogueWarp0 = 2;
inline constexpr int kReduceWarp0 = 6;
inline constexpr int kReduceWarps = 4;
// Warps that may run reduce / gather sub-tasks: the worker warps from the
// start, the epilogue warps once the GEMM queue is drained.
inline constexpr int kWorkerWarps = 8;
inline constexpr std::uint64_t kLocalTimeoutNs = 4000000000ull;

// kPair: the CTA of a 2-CTA cluster that computes one half of a 256-row pair
// tile; it stages its own 128 rows of A and half (BN / 2 columns) of B.
template <int BN, bool kPair = false>
struct gemm_config {
  static_assert(BN == 64 || BN == 128 || BN == 256, "tile_n must be 64, 128 or 256");
  static_assert(!kPair || BN >= 128, "CTA pairs need tile_n >= 128");
  static constexpr int b_cols = kPair ? BN / 2 : BN;          // B columns staged per CTA
  static constexpr int a_bytes = kBlockM * kBlockK * 2;        // 16 KiB
  static constexpr int b_panel_bytes = kBlockK * 64 * 2;       // 8 KiB per 64 columns
  static constexpr int b_bytes = kBlockK * b_cols * 2;
  static constexpr int stage_bytes = a_bytes + b_bytes;
  // Bytes one stage's full barrier waits for (the leader's counts both CTAs).
  static constexpr int tx_bytes = kPair ? 2 * stage_bytes : stage_bytes;
  static constexpr int stages = (192 * 1024) / stage_bytes;    // 4 / 6 / 8; pairs 8 / 6
  static constexpr int ring_bytes = stages * stage_bytes;      // 192 KiB
  // One CTA per tile with fewer A rows than 128 (one tile row, m < 128): each
  // TMA load brings only the first a_box_rows rows of A, a stage shrinks to
  // a_box_rows * 128 B + b_bytes, and up to max_stages such stages fit the
  // same ring (the MMA still reads 128 rows; rows past a_box_rows hold
  // whatever lies there and only produce accumulator rows that are never
  // stored).
  static constexpr int max_stages = kPair ? stages : 24;
  static constexpr int col_blocks = BN / 64;                   // sub-tasks per quarter
  static constexpr int reduce_bytes = kWorkerWarps * 32 * 128; // transpose tiles
  static constexpr int n_barriers = 2 * max_stages + 4 + 2 * kTaskRing + 3;
  static constexpr int aux_bytes = n_barriers * 8 + kTaskRing * 4 + 16;
  static constexpr int smem_bytes = 1024 + ring_bytes + reduce_bytes + aux_bytes;
  static_assert(smem_bytes <= 232448, "dynamic shared memory per CTA");
  static constexpr int tmem_columns = 2 * BN;
};

struct gemm_ar_params {
  std::int32_t m, n, k;
  std::int32_t m_tiles, n_tiles, tiles;
  std::int32_t n_pes, my_pe;
  std::int32_t mode;          // mode_allreduce / mode_reduce_scatter
  std::int32_t one_shot;      // 1: every PE reduces every tile
  std::int32_t group_m;
  std::int32_t n_comm;        // communication sub-tasks (reduced tiles x quarters)
  std::int32_t comm_warps;    // warps per CTA running them: the last comm_warps of 2..9
  std::int32_t rows_per_pe;   // reduce-scatter: output rows per PE
  std::uint64_t timeout_ns;   // bound of cross-GPU waits
  __nv_bfloat16 *out;         // this PE's output
  char *workspace;            // this PE's partial slots (symmetric)
  std::uint32_t *events;      // this PE's events buffer (symmetric)
  // In-switch reduction (two-shot bf16 allreduce with workspace and out in
  // the team's multicast region): their multicast addresses; else null.
  char *mc_workspace;
  __nv_bfloat16 *mc_out;
  megacu::nvshmem::peer_table peers;
  unsigned long long *trace;
  std::int64_t trace_capacity;
  // All-gather + GEMM (mode_allgather): this PE's A shard [rows_per_pe, k]
  // (symmetric: the peers copy it), the gathered A [m, k] (local), and the
  // copy chunking: chunk_rows whole rows per chunk, chunks_per_block chunks
  // per 128-row tile row (n_comm = n_pes * tile rows per shard * that).
  __nv_bfloat16 const *a_shard;
  __nv_bfloat16 *gathered;
  std::int32_t chunk_rows;
  std::int32_t chunks_per_block;
  // Rows of A one TMA load brings: 0 or 128 = a whole tile; fewer (a
  // multiple of 8, covering m) for one tile row without CTA pairs, so that
  // more, smaller stages hide the load latency (map_a's box has this height).
  std::int32_t a_box_rows;
  // 0 or 1: one CTA per tile. 2 or 4 (one tile row, no CTA pairs, launched as
  // clusters of that size, at most one tile per cluster): the cluster's CTAs
  // compute the same tile over consecutive ranges of K and rank 0 adds the
  // others' accumulators (received in its stage ring through distributed
  // shared memory) before its epilogue.
  std::int32_t k_split;
  // 1: one-shot peer exchange of one tile row (decode shapes, bf16 wire):
  // sub-tasks are 16-column slices of a block (comm_tasks_slices), so that a
  // warp loads one slice from every PE in one round trip.
  std::int32_t comm_slices;
};

namespace detail {

__device__ __forceinline__ control_block *control(gemm_ar_params const &p) {
  return reinterpret_cast<control_block *>(p.events);
}

__device__ __forceinline__ std::uint32_t *event_words(std::uint32_t *events) {
  return reinterpret_cast<std::uint32_t *>(reinterpret_cast<char *>(events) + kControlBytes);
}

__device__ __forceinline__ void record_error(gemm_ar_params const &p, std::uint32_t code,
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

__device__ __forceinline__ void count(gemm_ar_params const &p, int which,
                                      unsigned long long v) {
  atomicAdd(&control(p)->counters[which], v);
}

// Optional trace record {kind | sub << 8 | CTA << 16 | ticket << 32, tile,
// start ns, end ns} (%globaltimer). Kinds: 0 GEMM tile (epilogue span),
// 2 reduce sub-task (after its acquire), 3 a worker's completion fence
// (ticket = its place among the finished workers), 4 this PE's done flags
// stored, 5 the wait for every PE's done flag, 6 an all-gather copy chunk
// (sub = how many PEs away its shard is, tile = shard * tile rows per
// shard + tile row).
__device__ __forceinline__ void trace(gemm_ar_params const &p, std::uint32_t kind,
                                      std::uint32_t sub, std::uint32_t ticket,
                                      std::uint32_t tile, std::uint64_t t0) {
  if (p.trace == nullptr) {
    return;
  }
  std::uint32_t const i = atomicAdd(&control(p)->trace_count, 1u);
  if (static_cast<std::int64_t>(i) >= p.trace_capacity) {
    return;
  }
  unsigned long long *rec = p.trace + static_cast<std::int64_t>(i) * 4;
  rec[0] = static_cast<unsigned long long>(kind) | (static_cast<unsigned long long>(sub) << 8) |
           (static_cast<unsigned long long>(blockIdx.x) << 16) |
           (static_cast<unsigned long long>(ticket) << 32);
  rec[1] = tile;
  rec[2] = t0;
  rec[3] = ptx::now_ns();
}

// Waits until `*flag == want`, polling relaxed with a short back-off and
// finishing with one system-scope acquire load. Gives up when the abort word
// is set or `timeout_ns` elapses.
__device__ __forceinline__ bool wait_flag(std::uint32_t const *flag, std::uint32_t want,
                                          std::uint32_t const *abort_word,
                                          std::uint64_t timeout_ns) {
  if (ptx::ld_acquire_sys(flag) == want) {
    return true;
  }
  std::uint64_t const start = ptx::now_ns();
  for (std::uint32_t spin = 1;; ++spin) {
    __nanosleep(spin < 64 ? 32 : 256);
    if (ptx::ld_relaxed_sys(flag) == want && ptx::ld_acquire_sys(flag) == want) {
      return true;
    }
    if ((spin & 15u) == 0) {
      if (ptx::ld_relaxed_gpu(abort_word) != 0) {
        return false;
      }
      if (ptx::now_ns() - start > timeout_ns) {
        return false;
      }
    }
  }
}

// Byte offset of this PE's partial slot (parity, tile) in its workspace.
__device__ __forceinline__ std::int64_t slot_offset(std::uint32_t parity, std::int32_t tile,
                                                    std::int32_t tiles, std::int64_t slot_bytes) {
  return (static_cast<std::int64_t>(parity) * tiles + tile) * slot_bytes;
}

// Does the 32-row quarter q x 64-column block c of tile (row, col) hold any
// output element?
template <int BN>
__device__ __forceinline__ bool block_exists(gemm_ar_params const &p, std::int32_t tile_row,
                                             std::int32_t tile_col, std::int32_t quarter,
                                             std::int32_t block) {
  return tile_row * kBlockM + quarter * 32 < p.m && tile_col * BN + block * 64 < p.n;
}

__device__ __forceinline__ std::uint32_t draw_ticket(std::uint32_t *counter, std::uint32_t lane) {
  std::uint32_t ticket = 0;
  if (lane == 0) ticket = atomicAdd(counter, 1u);
  return __shfl_sync(0xffffffffu, ticket, 0);
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], uint4 w) {
  acc[0] += ptx::bf16_lo(w.x);
  acc[1] += ptx::bf16_hi(w.x);
  acc[2] += ptx::bf16_lo(w.y);
  acc[3] += ptx::bf16_hi(w.y);
  acc[4] += ptx::bf16_lo(w.z);
  acc[5] += ptx::bf16_hi(w.z);
  acc[6] += ptx::bf16_lo(w.w);
  acc[7] += ptx::bf16_hi(w.w);
}

// Communication worker (task 2): one warp takes sub-tasks = (reduced tile,
// 32-row quarter, 64-column block) in raster order from the reduce queue
// until it is empty; the reduced tiles are this PE's own (two-shot allreduce,
// reduce-scatter) or all of them (one-shot). For each: acquire every PE's
// arrive flag of the quarter, load the block of every PE's partial slot (its
// own memory for this PE, NVLink for the others), sum in PE order
// 0..n_pes-1 in fp32 (two PEs' loads in flight at a time), round to bf16,
// transpose 32 x 64 through `xpose` (4 KiB of shared memory) and store it
// row-major into this PE's out — in two-shot allreduce into every PE's out.
// Those stores are not flagged one by one: when the queue is empty the warp
// fences once, and the last worker of this PE announces "all my blocks are
// written" to every PE (finish_pushes).
template <int BN, bool kWireF32>
__device__ __forceinline__ void comm_tasks_peer(gemm_ar_params const &p, tile_schedule const &sched,
                                           std::uint32_t parity, std::uint32_t epoch,
                                           std::uint32_t *my_events,
                                           std::uint32_t const *abort_word, std::uint8_t *xpose,
                                           std::uint32_t lane) {
  constexpr int kWireBytes = kWireF32 ? 4 : 2;
  constexpr int kBlocks = BN / 64;
  constexpr std::int64_t kSlotBytes = std::int64_t(kBlockM) * BN * kWireBytes;
  constexpr std::int64_t kVecStride = kBlockM * 16;  // bytes between wire vectors of a row
  control_block *ctrl = control(p);
  bool const push_all = p.mode == mode_allreduce && !p.one_shot;
  for (;;) {
    std::uint32_t const ticket = draw_ticket(&ctrl->reduce_ticket, lane);
    if (ticket >= static_cast<std::uint32_t>(p.n_comm)) {
      break;
    }
    std::int32_t const j = static_cast<std::int32_t>(ticket) / (kQuarters * kBlocks);
    std::int32_t const rem = static_cast<std::int32_t>(ticket) % (kQuarters * kBlocks);
    std::int32_t const quarter = rem / kBlocks;
    std::int32_t const cb = rem % kBlocks;
    std::int32_t const r = p.one_shot ? j : j * p.n_pes + p.my_pe;
    tile_coord const c = locate(sched, r);
    std::int32_t const tile = c.tile_row * p.n_tiles + c.tile_col;
    if (!block_exists<BN>(p, c.tile_row, c.tile_col, quarter, cb)) {
      continue;  // no output element lives in this block
    }

    // Task 2 "before": every PE's partial of this quarter is ready.
    bool ok = true;
    if (static_cast<std::int32_t>(lane) < p.n_pes) {
      ok = wait_flag(my_events + arrive_index(parity, lane, tile, quarter, p.n_pes, p.tiles),
                     epoch, abort_word, p.timeout_ns);
      if (!ok) record_error(p, err_remote_timeout, tile, lane, 8);
    }
    if (!__all_sync(0xffffffffu, ok)) {
      break;
    }
    __syncwarp();  // orders every lane's loads after the lanes' acquires
    std::uint64_t const t0 = ptx::now_ns();

    float acc[8][8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] = 0.0f;
    }
    // Lane = row of the quarter; vector (v, row) of a slot at (v * 128 + row) * 16.
    std::int64_t const in_slot = slot_offset(parity, tile, p.tiles, kSlotBytes) +
                                 (static_cast<std::int64_t>(quarter) * 32 + lane) * 16;
    if constexpr (kWireF32) {
#pragma unroll 1
      for (std::int32_t src = 0; src < p.n_pes; ++src) {
        char const *base = p.peers.translate(p.workspace, src) + in_slot;
        uint4 w[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) w[h] = ptx::ld_cg_v4(base + (cb * 16 + h) * kVecStride);
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          acc[h / 2][(h % 2) * 4 + 0] += __uint_as_float(w[h].x);
          acc[h / 2][(h % 2) * 4 + 1] += __uint_as_float(w[h].y);
          acc[h / 2][(h % 2) * 4 + 2] += __uint_as_float(w[h].z);
          acc[h / 2][(h % 2) * 4 + 3] += __uint_as_float(w[h].w);
        }
      }
    } else {
#pragma unroll 1
      for (std::int32_t src = 0; src < p.n_pes; src += 2) {
        bool const pair = src + 1 < p.n_pes;
        char const *base0 = p.peers.translate(p.workspace, src) + in_slot;
        uint4 w0[8], w1[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) w0[g] = ptx::ld_cg_v4(base0 + (cb * 8 + g) * kVecStride);
        if (pair) {
          char const *base1 = p.peers.translate(p.workspace, src + 1) + in_slot;
#pragma unroll
          for (int g = 0; g < 8; ++g) w1[g] = ptx::ld_cg_v4(base1 + (cb * 8 + g) * kVecStride);
        }
#pragma unroll
        for (int g = 0; g < 8; ++g) add_bf16x8(acc[g], w0[g]);
        if (pair) {
#pragma unroll
          for (int g = 0; g < 8; ++g) add_bf16x8(acc[g], w1[g]);
        }
      }
    }
    // Row `lane` of the 32 x 64 block -> shared, 16 B per 8 columns,
    // XOR-swizzled so that both the write and the read are conflict-free.
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
    // Read back row-major: 8 lanes cover one 128 B row segment.
    std::int32_t const row0 = c.tile_row * kBlockM + quarter * 32;
    std::int32_t const out_row0 =
        p.mode == mode_reduce_scatter ? row0 - c.owner * p.rows_per_pe : row0;
    std::int32_t const g = lane % 8;
    std::int32_t const col = c.tile_col * BN + cb * 64 + g * 8;
    // Every PE's out in two-shot allreduce (one multicast store each with
    // the in-switch reduction; else starting with the next PE, so the PEs
    // spread their stores over the links), this PE's out otherwise.
    std::int32_t const n_out = push_all ? p.n_pes : 1;
    for (std::int32_t d = 0; d < n_out; ++d) {
      std::int32_t const pe = push_all ? (p.my_pe + 1 + d) % p.n_pes : p.my_pe;
      __nv_bfloat16 *dst = push_all ? p.peers.translate(p.out, pe) : p.out;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        std::int32_t const rr = i * 4 + static_cast<std::int32_t>(lane) / 8;
        uint4 const q = *reinterpret_cast<uint4 const *>(xpose + rr * 128 + ((g ^ (rr & 7)) * 16));
        if (row0 + rr < p.m && col < p.n) {
          ptx::st_v4(dst + static_cast<std::int64_t>(out_row0 + rr) * p.n + col, q);
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      count(p, ctr_reduce_tasks, 1);
      count(p, ctr_partial_acquire, p.n_pes);
      if (push_all) count(p, ctr_final_publish, p.n_pes);
      trace(p, 2, quarter * kBlocks + cb, ticket, tile, t0);
    }
  }
}

// One-shot peer exchange of one tile row (decode shapes, bf16 wire): the few
// blocks such a call has leave most worker warps idle, while a block summed
// by one warp takes one NVLink round trip per pair of PEs. Here a sub-task is
// (tile, 32-row quarter, 64-column block, 16-column slice): a warp acquires
// the quarter's flags, loads its slice (two 16-byte vectors per row) from every
// PE at once, sums in PE order 0..n_pes-1 in fp32 (the same sum as
// comm_tasks_peer), rounds once to bf16 and stores its rows into this PE's
// out. Counters and trace records are kept per block (slice 0), as the task
// graph counts them.
template <int BN>
__device__ __forceinline__ void comm_tasks_slices(gemm_ar_params const &p,
                                                  tile_schedule const &sched,
                                                  std::uint32_t parity, std::uint32_t epoch,
                                                  std::uint32_t *my_events,
                                                  std::uint32_t const *abort_word,
                                                  std::uint32_t lane) {
  constexpr int kBlocks = BN / 64;
  constexpr int kSlices = 4;                          // 16 columns each
  constexpr std::int64_t kSlotBytes = std::int64_t(kBlockM) * BN * 2;
  constexpr std::int64_t kVecStride = kBlockM * 16;  // bytes between wire vectors of a row
  constexpr int kMaxPes = megacu::nvshmem::max_team_pes;
  control_block *ctrl = control(p);
  for (;;) {
    std::uint32_t const ticket = draw_ticket(&ctrl->reduce_ticket, lane);
    if (ticket >= static_cast<std::uint32_t>(p.n_comm)) {
      break;
    }
    std::int32_t const j = static_cast<std::int32_t>(ticket) / (kQuarters * kBlocks * kSlices);
    std::int32_t const rem = static_cast<std::int32_t>(ticket) % (kQuarters * kBlocks * kSlices);
    std::int32_t const quarter = rem / (kBlocks * kSlices);
    std::int32_t const cb = (rem / kSlices) % kBlocks;
    std::int32_t const sl = rem % kSlices;
    tile_coord const c = locate(sched, j);  // one-shot: every tile, raster order
    std::int32_t const tile = c.tile_row * p.n_tiles + c.tile_col;
    if (!block_exists<BN>(p, c.tile_row, c.tile_col, quarter, cb)) {
      continue;  // no output element lives in this block
    }
    bool ok = true;
    if (static_cast<std::int32_t>(lane) < p.n_pes) {
      ok = wait_flag(my_events + arrive_index(parity, lane, tile, quarter, p.n_pes, p.tiles),
                     epoch, abort_word, p.timeout_ns);
      if (!ok) record_error(p, err_remote_timeout, tile, lane, 8);
    }
    if (!__all_sync(0xffffffffu, ok)) {
      break;
    }
    __syncwarp();  // orders every lane's loads after the lanes' acquires
    std::uint64_t const t0 = ptx::now_ns();
    // Lane = row of the quarter; vector (v, row) of a slot at (v * 128 + row) * 16.
    std::int64_t const in_slot = slot_offset(parity, tile, p.tiles, kSlotBytes) +
                                 (static_cast<std::int64_t>(quarter) * 32 + lane) * 16 +
                                 static_cast<std::int64_t>(cb * 8 + sl * 2) * kVecStride;
    uint4 w[kMaxPes][2];
#pragma unroll
    for (int src = 0; src < kMaxPes; ++src) {
      if (src < p.n_pes) {
        char const *base = p.peers.translate(p.workspace, src) + in_slot;
        w[src][0] = ptx::ld_cg_v4(base);
        w[src][1] = ptx::ld_cg_v4(base + kVecStride);
      }
    }
    float acc[2][8];
#pragma unroll
    for (int v = 0; v < 2; ++v) {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[v][e] = 0.0f;
    }
#pragma unroll
    for (int src = 0; src < kMaxPes; ++src) {
      if (src < p.n_pes) {
        add_bf16x8(acc[0], w[src][0]);
        add_bf16x8(acc[1], w[src][1]);
      }
    }
    std::int32_t const row = c.tile_row * kBlockM + quarter * 32 + static_cast<std::int32_t>(lane);
    std::int32_t const col = c.tile_col * BN + cb * 64 + sl * 16;
    if (row < p.m) {
      __nv_bfloat16 *at = p.out + static_cast<std::int64_t>(row) * p.n + col;
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        if (col + v * 8 < p.n) {
          uint4 q;
          q.x = ptx::pack_bf16x2(acc[v][0], acc[v][1]);
          q.y = ptx::pack_bf16x2(acc[v][2], acc[v][3]);
          q.z = ptx::pack_bf16x2(acc[v][4], acc[v][5]);
          q.w = ptx::pack_bf16x2(acc[v][6], acc[v][7]);
          ptx::st_v4(at + v * 8, q);
        }
      }
    }
    __syncwarp();
    if (lane == 0 && sl == 0) {
      count(p, ctr_reduce_tasks, 1);
      count(p, ctr_partial_acquire, p.n_pes);
      trace(p, 2, quarter * kBlocks + cb, ticket, tile, t0);
    }
  }
}

// In-switch reduction worker (task 2 with the workspace in the team's
// multicast region, bf16 wire): one warp takes sub-tasks = (reduced tile,
// 32-row quarter) in raster order; the reduced tiles are this PE's own
// (two-shot allreduce, reduce-scatter) or all of them (one-shot). For each:
// acquire every PE's arrive flag of the quarter once, then for each 64-column
// block in order read the sum over every PE's slot with one
// `multimem.ld_reduce` per 16-byte vector (fp32 accumulation in the NVSwitch,
// one bf16 rounding), transpose 32 x 64 through `xpose` and store it
// row-major: in two-shot allreduce with one `multimem.st` per vector into
// every PE's out, else into this PE's out. Once a block is staged in shared
// memory the next block's loads are issued, so they are in flight while the
// block is stored; the next ticket is drawn while the current one runs.
template <int BN>
__device__ __forceinline__ void comm_tasks_switch(gemm_ar_params const &p,
                                                  tile_schedule const &sched,
                                                  std::uint32_t parity, std::uint32_t epoch,
                                                  std::uint32_t *my_events,
                                                  std::uint32_t const *abort_word,
                                                  std::uint8_t *xpose, std::uint32_t lane) {
  constexpr int kBlocks = BN / 64;
  constexpr std::int64_t kSlotBytes = std::int64_t(kBlockM) * BN * 2;
  constexpr std::int64_t kVecStride = kBlockM * 16;  // bytes between wire vectors of a row
  control_block *ctrl = control(p);
  bool const push_all = p.mode == mode_allreduce && !p.one_shot;  // then p.mc_out is set
  std::int32_t const g = static_cast<std::int32_t>(lane) % 8;      // 16 B column group of a row
  std::uint32_t ticket = draw_ticket(&ctrl->reduce_ticket, lane);
  while (ticket < static_cast<std::uint32_t>(p.n_comm)) {
    // Draw the next ticket now; its atomic completes while this one runs.
    std::uint32_t next_raw = 0;
    if (lane == 0) next_raw = atomicAdd(&ctrl->reduce_ticket, 1u);
    std::int32_t const j = static_cast<std::int32_t>(ticket) / kQuarters;
    std::int32_t const quarter = static_cast<std::int32_t>(ticket) % kQuarters;
    std::int32_t const r = p.one_shot ? j : j * p.n_pes + p.my_pe;
    tile_coord const c = locate(sched, r);
    std::int32_t const tile = c.tile_row * p.n_tiles + c.tile_col;
    // Blocks of this quarter that hold output elements: the first `blocks`.
    std::int32_t blocks = 0;
#pragma unroll
    for (int cb = 0; cb < kBlocks; ++cb) {
      blocks += block_exists<BN>(p, c.tile_row, c.tile_col, quarter, cb) ? 1 : 0;
    }
    if (blocks == 0) {  // no output element lives in this quarter
      ticket = __shfl_sync(0xffffffffu, next_raw, 0);
      continue;
    }
    // Task 2 "before": every PE's partial of this quarter is ready.
    bool ok = true;
    if (static_cast<std::int32_t>(lane) < p.n_pes) {
      ok = wait_flag(my_events + arrive_index(parity, lane, tile, quarter, p.n_pes, p.tiles),
                     epoch, abort_word, p.timeout_ns);
      if (!ok) record_error(p, err_remote_timeout, tile, lane, 8);
    }
    if (!__all_sync(0xffffffffu, ok)) {
      break;
    }
    __syncwarp();  // orders every lane's loads after the lanes' acquires
    std::uint64_t const t0 = ptx::now_ns();
    // Lane = row of the quarter; vector (v, row) of a slot at (v * 128 + row) * 16.
    char const *mc = p.mc_workspace + slot_offset(parity, tile, p.tiles, kSlotBytes) +
                     (static_cast<std::int64_t>(quarter) * 32 + lane) * 16;
    std::int32_t const row0 = c.tile_row * kBlockM + quarter * 32;
    std::int32_t const out_row0 =
        p.mode == mode_reduce_scatter ? row0 - c.owner * p.rows_per_pe : row0;
    uint4 w[8];
#pragma unroll
    for (int gg = 0; gg < 8; ++gg) w[gg] = ptx::multimem_ld_reduce_bf16x8(mc + gg * kVecStride);
#pragma unroll 1
    for (int cb = 0; cb < blocks; ++cb) {
      // Row `lane` of the block -> shared memory, 16 B per 8 columns,
      // XOR-swizzled so that both the write and the read are conflict-free.
#pragma unroll
      for (int gg = 0; gg < 8; ++gg) {
        *reinterpret_cast<uint4 *>(xpose + lane * 128 + ((gg ^ (lane & 7)) * 16)) = w[gg];
      }
      __syncwarp();
      if (cb + 1 < blocks) {
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
          w[gg] = ptx::multimem_ld_reduce_bf16x8(mc + ((cb + 1) * 8 + gg) * kVecStride);
        }
      }
      // Read back row-major: 8 lanes cover one 128 B row segment.
      std::int32_t const col = c.tile_col * BN + cb * 64 + g * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        std::int32_t const rr = i * 4 + static_cast<std::int32_t>(lane) / 8;
        uint4 const q =
            *reinterpret_cast<uint4 const *>(xpose + rr * 128 + ((g ^ (rr & 7)) * 16));
        if (row0 + rr < p.m && col < p.n) {
          std::int64_t const at = static_cast<std::int64_t>(out_row0 + rr) * p.n + col;
          if (push_all) {
            ptx::multimem_st_v4(p.mc_out + at, q);
          } else {
            ptx::st_v4(p.out + at, q);
          }
        }
      }
      __syncwarp();  // every lane has read xpose before the next block writes it
    }
    if (lane == 0) {
      count(p, ctr_reduce_tasks, static_cast<unsigned long long>(blocks));
      count(p, ctr_partial_acquire, static_cast<unsigned long long>(blocks) * p.n_pes);
      if (push_all) count(p, ctr_final_publish, static_cast<unsigned long long>(blocks) * p.n_pes);
      trace(p, 2, static_cast<std::uint32_t>(quarter), ticket, tile, t0);
    }
    ticket = __shfl_sync(0xffffffffu, next_raw, 0);
  }
}

// Two-shot allreduce completion. Each worker warp, once the reduce queue is
// empty, fences its stores at system scope (they went to every PE's out,
// directly or through the multicast object) and
// counts itself done; the last worker of this PE then sets done[p][my_pe] on
// every PE. One system-scope fence per warp per call instead of one per block.
__device__ __forceinline__ void finish_pushes(gemm_ar_params const &p, std::uint32_t parity,
                                              std::uint32_t epoch, std::uint32_t *my_events,
                                              std::uint32_t lane) {
  control_block *ctrl = control(p);
  std::uint64_t const t0 = ptx::now_ns();
  if (p.mc_out != nullptr) {
    ptx::fence_proxy_alias();  // the stores went through the multicast mapping
  }
  ptx::fence_acq_rel_sys();
  __syncwarp();
  std::uint32_t last = 0;
  if (lane == 0) {
    std::uint32_t const total = gridDim.x * static_cast<std::uint32_t>(p.comm_warps);
    std::uint32_t const done = atomicAdd(&ctrl->workers_done, 1u);
    last = done == total - 1 ? 1u : 0u;
    trace(p, 3, 0, done, 0, t0);
  }
  if (__shfl_sync(0xffffffffu, last, 0) == 0) {
    return;
  }
  std::uint64_t const t1 = ptx::now_ns();
  ptx::fence_acq_rel_sys();
  if (static_cast<std::int32_t>(lane) < p.n_pes) {
    std::uint32_t *flags = p.peers.translate(my_events, lane);
    ptx::st_relaxed_sys(flags + done_index(parity, p.my_pe, p.n_pes, p.tiles), epoch);
  }
  __syncwarp();
  if (lane == 0) trace(p, 4, 0, 0, 0, t1);
}

// Two-shot allreduce: this PE's out is complete once every PE has announced
// that all of its blocks are written (one waiter per PE suffices: the launch
// ends only when this warp does).
__device__ __forceinline__ void wait_all_pushes(gemm_ar_params const &p, std::uint32_t parity,
                                                std::uint32_t epoch, std::uint32_t *my_events,
                                                std::uint32_t const *abort_word,
                                                std::uint32_t lane) {
  bool ok = true;
  std::uint64_t const t0 = ptx::now_ns();
  if (static_cast<std::int32_t>(lane) < p.n_pes) {
    ok = wait_flag(my_events + done_index(parity, lane, p.n_pes, p.tiles), epoch, abort_word,
                   p.timeout_ns);
    if (!ok) record_error(p, err_remote_timeout, 0xffffffffu, lane, 9);
  }
  bool const all = __all_sync(0xffffffffu, ok);
  if (lane == 0 && all) {
    count(p, ctr_final_acquire, p.n_pes);
    trace(p, 5, 0, 0, 0, t0);
  }
}

// Waits until the local counter `*counter` reaches `target` (acquire at GPU
// scope), or gives up when the abort word is set or `timeout_ns` elapses.
__device__ __forceinline__ bool wait_at_least(std::uint32_t const *counter, std::uint32_t target,
                                              std::uint32_t const *abort_word,
                                              std::uint64_t timeout_ns) {
  if (ptx::ld_acquire_gpu(counter) >= target) {
    return true;
  }
  std::uint64_t const start = ptx::now_ns();
  for (std::uint32_t spin = 1;; ++spin) {
    __nanosleep(spin < 64 ? 32 : 256);
    if (ptx::ld_relaxed_gpu(counter) >= target && ptx::ld_acquire_gpu(counter) >= target) {
      return true;
    }
    if ((spin & 15u) == 0) {
      if (ptx::ld_relaxed_gpu(abort_word) != 0) {
        return false;
      }
      if (ptx::now_ns() - start > timeout_ns) {
        return false;
      }
    }
  }
}

// All-gather worker: one warp takes copy chunks from the gather queue (the
// reduce ticket) until it is empty. Ticket t = (slot, tile row rb of the
// shard, chunk j of the row); slot s copies the shard of the PE s + 1 hops
// away, the last slot this PE's own shard, so peers' rows arrive in the
// order the GEMM raster needs them and the PEs start on different sources.
// A chunk is chunk_rows whole rows of the source shard (one contiguous
// range), loaded over NVLink (or locally) and stored into those rows of the
// gathered A. The first chunk a warp takes from a shard waits for the
// shard's ready flag. After each chunk the tile row's counter is raised with
// a GPU-scope release (this PE's GEMM producer acquires it before its TMA
// loads), and the warp that completes a peer's shard tells that peer.
__device__ __forceinline__ void gather_tasks(gemm_ar_params const &p, std::uint32_t epoch,
                                             std::uint32_t *my_events, gather_words const &gw,
                                             std::uint32_t const *abort_word,
                                             std::uint32_t lane) {
  control_block *ctrl = control(p);
  std::int32_t const per_block = p.chunks_per_block;
  std::int32_t const per_shard = gw.mq * per_block;  // chunks of one shard
  std::int64_t const chunk_vecs = static_cast<std::int64_t>(p.chunk_rows) * p.k / 8;
  std::uint32_t seen = 0;  // bit src: src's ready flag acquired by this warp
  for (;;) {
    std::uint32_t const ticket = draw_ticket(&ctrl->reduce_ticket, lane);
    if (ticket >= static_cast<std::uint32_t>(p.n_comm)) {
      break;
    }
    gather_chunk const ch = locate_gather_chunk(static_cast<std::int32_t>(ticket), p.n_pes,
                                                p.my_pe, gw.mq, per_block, p.chunk_rows);
    std::int32_t const rb = ch.rb;
    std::int32_t const hops = ch.hops;
    std::int32_t const src = ch.src;
    bool const remote = src != p.my_pe;
    if constexpr (kCheckBounds) {
      bool const in = src >= 0 && src < p.n_pes && rb >= 0 && rb < gw.mq && ch.row0 >= 0 &&
                      ch.row0 + p.chunk_rows <= p.rows_per_pe &&
                      static_cast<std::int64_t>(src) * p.rows_per_pe + ch.row0 + p.chunk_rows <=
                          p.m &&
                      gw.chunks(src) < gw.end();
      if (!in) {
        if (lane == 0) record_error(p, err_bounds, ticket, static_cast<std::uint32_t>(src), 30);
        continue;  // nothing copied or counted: the tiles waiting on it time out
      }
    }
    if (remote && ((seen >> src) & 1u) == 0) {
      bool ok = true;
      if (lane == 0) {
        ok = wait_flag(my_events + gw.ready(src), epoch, abort_word, p.timeout_ns);
        if (!ok) record_error(p, err_remote_timeout, static_cast<std::uint32_t>(rb),
                              static_cast<std::uint32_t>(src), 21);
      }
      if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0) {
        break;
      }
      seen |= 1u << src;
    }
    __syncwarp();  // every lane's loads after lane 0's acquire
    std::uint64_t const t0 = ptx::now_ns();
    std::int64_t const row0 = ch.row0;
    __nv_bfloat16 const *shard = remote ? p.peers.translate(p.a_shard, src) : p.a_shard;
    auto const *from = reinterpret_cast<uint4 const *>(shard + row0 * p.k);
    auto *to = reinterpret_cast<uint4 *>(
        p.gathered + (static_cast<std::int64_t>(src) * p.rows_per_pe + row0) * p.k);
    // Eight 512-byte warp loads in flight, then their stores.
    for (std::int64_t v0 = 0; v0 < chunk_vecs; v0 += 8 * 32) {
      uint4 w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        std::int64_t const v = v0 + u * 32 + lane;
        w[u] = v < chunk_vecs ? ptx::ld_cg_v4(from + v) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        std::int64_t const v = v0 + u * 32 + lane;
        if (v < chunk_vecs) ptx::st_v4(to + v, w[u]);
      }
    }
    ptx::fence_acq_rel_gpu();
    __syncwarp();
    if (lane == 0) {
      ptx::red_release_gpu_add(my_events + gw.rows(src, rb), 1u);
      std::uint32_t const done = atomicAdd(my_events + gw.chunks(src), 1u);
      if (remote && done + 1 == static_cast<std::uint32_t>(per_shard)) {
        // Every chunk of src's shard is copied (the other warps' loads are
        // ordered before their counts): src may overwrite its shard after
        // this call.
        ptx::fence_acq_rel_sys();
        ptx::st_relaxed_sys(p.peers.translate(my_events, src) + gw.read_done(p.my_pe), epoch);
        count(p, ctr_final_publish, 1);
      }
      count(p, ctr_reduce_tasks, 1);
      trace(p, 6, static_cast<std::uint32_t>(hops), ticket,
            static_cast<std::uint32_t>(src * gw.mq + rb), t0);
    }
  }
}

// All-gather: the call ends only after every peer has copied this PE's
// shard, so no later write to the shard (stream-ordered after this call)
// can race a peer's read of it.
__device__ __forceinline__ void wait_all_reads(gemm_ar_params const &p, std::uint32_t epoch,
                                               std::uint32_t *my_events, gather_words const &gw,
                                               std::uint32_t const *abort_word,
                                               std::uint32_t lane) {
  bool ok = true;
  std::int32_t const pe = static_cast<std::int32_t>(lane);
  if (pe < p.n_pes && pe != p.my_pe) {
    ok = wait_flag(my_events + gw.read_done(pe), epoch, abort_word, p.timeout_ns);
    if (!ok) record_error(p, err_remote_timeout, 0xffffffffu, lane, 22);
  }
  if (__all_sync(0xffffffffu, ok) && lane == 0) {
    count(p, ctr_final_acquire, static_cast<unsigned long long>(p.n_pes - 1));
  }
}

}  // namespace detail

// Bounded mbarrier wait; CTA-pair kernels wait with cluster-scope acquire
// because the other CTA of the pair arrives on some of their barriers.
template <bool kPair>
__device__ __forceinline__ bool bar_wait(std::uint64_t *bar, std::uint32_t parity,
                                         std::uint32_t const *abort_word,
                                         std::uint64_t timeout_ns = kLocalTimeoutNs) {
  if constexpr (kPair) {
    return ptx::mbar_wait_cluster(bar, parity, abort_word, timeout_ns);
  } else {
    return ptx::mbar_wait(bar, parity, abort_word, timeout_ns);
  }
}

// kPair = false: one CTA per SM, each GEMM ticket is one 128 x BN tile.
// kPair = true: launched as 2-CTA clusters; each GEMM ticket is a 256 x BN
// pair tile computed by both CTAs with cta_group::2 MMAs issued by the
// leader (cluster rank 0). Each CTA TMA-loads its own 128 rows of A and its
// half of B into its own shared memory (completion counted on the leader's
// full barrier), and holds its 128 accumulator rows in its own TMEM, so the
// epilogue and everything after it are the same in both CTAs. The leader
// relays the barrier events the follower needs (stage free, accumulator
// ready, next task) with remote mbarrier arrives; the follower reports back
// (task taken, accumulator drained) the same way.
//
// kGather = true: all-gather + GEMM (mode_allgather). `map_a` is this PE's
// A shard, `map_b2` the gathered A [m, k]; tiles of this PE's own shard read
// the shard, the others the gathered rows once their tile row's counter says
// every chunk is copied. The epilogue stores the tile into this PE's out
// (local) and marks its quarters in the arrive plane, as one PE would; the
// workers run the copies (gather_tasks) instead of reductions.
//
// kSwiGLU = true (one PE, no exchange): the gate/up projection of an MLP
// block. A tile's BN accumulator columns are BN/2 gate columns (B panels from
// `map_b`) followed by the same BN/2 columns of up (`map_b2`; with pairs the
// leader stages gate, the follower up); the epilogue stores
// silu(gate) * up as bf16 into out[m, n] (n = the act columns, tiles of
// BN/2). Otherwise `map_b2` is unused.
template <int BN, bool kWireF32, bool kPair = false, bool kSwiGLU = false, bool kGather = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_ar_megakernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_b2,
                       const __grid_constant__ gemm_ar_params p) {
  static_assert(!kSwiGLU || (BN == 256 && !kWireF32), "SwiGLU tiles are 128 x (128 + 128)");
  static_assert(!kGather || (!kSwiGLU && !kWireF32), "all-gather tiles are plain bf16 tiles");
  using cfg = gemm_config<BN, kPair>;
  constexpr int kWireBytes = kWireF32 ? 4 : 2;
  constexpr int kVecCols = 16 / kWireBytes;                   // columns per 16 B wire vector
  constexpr std::int64_t kSlotBytes = std::int64_t(kBlockM) * BN * kWireBytes;

  extern __shared__ std::uint8_t smem_raw[];
  std::uint32_t const raw_addr = ptx::smem_addr(smem_raw);
  std::uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  std::uint8_t *stages = smem;
  std::uint8_t *reduce_smem = smem + cfg::ring_bytes;
  auto *bars = reinterpret_cast<std::uint64_t *>(reduce_smem + cfg::reduce_bytes);
  std::uint64_t *full = bars;
  std::uint64_t *empty = full + cfg::max_stages;
  std::uint64_t *acc_full = empty + cfg::max_stages;
  std::uint64_t *acc_empty = acc_full + 2;
  std::uint64_t *task_full = acc_empty + 2;
  std::uint64_t *task_empty = task_full + kTaskRing;
  std::uint64_t *mma_done = task_empty + kTaskRing;
  std::uint64_t *ring_free = mma_done + 1;  // K split: rank 0's stage ring may be written
  std::uint64_t *recv_full = ring_free + 1; // K split: the other ranks' accumulators arrived
  auto *ring = reinterpret_cast<std::int32_t volatile *>(recv_full + 1);
  auto *tmem_slot = reinterpret_cast<std::uint32_t *>(const_cast<std::int32_t *>(ring) + kTaskRing);
  auto *epoch_slot = tmem_slot + 1;

  int const warp = threadIdx.x / 32;
  std::uint32_t const lane = threadIdx.x % 32;
  control_block *ctrl = detail::control(p);
  std::uint32_t const *abort_word = &ctrl->error_code;
  tile_schedule const sched{p.m_tiles, p.n_tiles, p.n_pes, p.mode, p.group_m,
                            kGather ? p.my_pe : 0};
  gather_words const gw = gather_layout(p.n_pes, p.tiles, p.m_tiles / p.n_pes);
  // Bound of the GEMM pipeline's waits. All-gather tiles wait for rows that
  // come from other GPUs, so there a stage may stay empty as long as a
  // cross-GPU wait may last.
  std::uint64_t const pipe_timeout = kGather ? p.timeout_ns + kLocalTimeoutNs : kLocalTimeoutNs;
  std::int32_t const k_blocks = (p.k + kBlockK - 1) / kBlockK;
  // GEMM tickets: tiles, or pair tiles.
  std::int32_t const gemm_units = kPair ? p.tiles / 2 : p.tiles;
  std::uint32_t const cta_rank = kPair ? ptx::cluster_ctarank() : 0u;
  bool const leader = cta_rank == 0;
  // Raster index of the tile this CTA computes for GEMM ticket q.
  auto tile_of = [&](std::int32_t q) {
    return kPair ? pair_raster(sched, q, static_cast<std::int32_t>(cta_rank)) : q;
  };
  // Stage ring: rows of A per load, bytes per stage and stages (see
  // gemm_config::max_stages); stage bases stay 1024-byte aligned.
  std::int32_t const a_rows = (!kPair && p.a_box_rows > 0) ? p.a_box_rows : kBlockM;
  std::uint32_t const a_bytes = static_cast<std::uint32_t>(a_rows) * 128u;
  std::uint32_t const stage_bytes = kPair ? cfg::stage_bytes : a_bytes + cfg::b_bytes;
  std::uint32_t const n_stages =
      kPair ? cfg::stages
            : (cfg::ring_bytes / stage_bytes < static_cast<std::uint32_t>(cfg::max_stages)
                   ? cfg::ring_bytes / stage_bytes
                   : static_cast<std::uint32_t>(cfg::max_stages));
  std::uint32_t const tx_bytes = kPair ? cfg::tx_bytes : stage_bytes;
  // K split over a cluster (gemm_ar_params::k_split): this CTA's rank and its
  // k-blocks [kb_begin, kb_end) (the host keeps k_blocks >= k_split).
  std::int32_t const k_split = (!kPair && p.k_split > 1) ? p.k_split : 1;
  std::uint32_t const split_rank = k_split > 1 ? ptx::cluster_ctarank() : 0u;
  std::int32_t const kb_begin = static_cast<std::int32_t>(split_rank) * k_blocks / k_split;
  std::int32_t const kb_end = (static_cast<std::int32_t>(split_rank) + 1) * k_blocks / k_split;
  // Single-CTA plain tiles: the first ticket is static, so thread 0 (the
  // producer) issues the first tile's first `pre_issued` stage loads right
  // after setting up the barriers, and the rest of the set-up (TMEM
  // allocation, block and cluster barriers) overlaps their latency. The
  // producer's loop then starts past them.
  constexpr bool kEarlyLoads = !kPair && !kSwiGLU && !kGather;
  std::uint32_t pre_issued = 0;

  if (threadIdx.x == 0) {
    // The launch counter and the tensor maps are fetched first, so that their
    // latency overlaps the barrier set-up below.
    std::uint32_t const launches = ptx::ld_relaxed_gpu(&ctrl->launch_count);
    ptx::prefetch_tensor_map(&map_a);
    ptx::prefetch_tensor_map(&map_b);
    if constexpr (kSwiGLU || kGather) ptx::prefetch_tensor_map(&map_b2);
    // Arrivals per phase. Pairs: the leader's acc_empty also counts the
    // follower's 4 epilogue warps, its task_empty the follower's 4 epilogue
    // warps and producer; the follower's own empty / acc_full / task_full
    // are arrived by the leader (one each).
    for (std::uint32_t s = 0; s < n_stages; ++s) {
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
    if (k_split > 1) {
      ptx::mbar_init(ring_free, 1);                            // rank 0's one arrive
      ptx::mbar_init(recv_full, 4 * static_cast<std::uint32_t>(k_split - 1));  // epilogue warps
    }
    ptx::fence_barrier_init();
    *epoch_slot = launches + 1u;
    if constexpr (kEarlyLoads) {
      // The first ticket exactly as the producer's loop takes it below.
      std::int32_t const first = static_cast<std::int32_t>(blockIdx.x) / k_split;
      std::int32_t const kbs = kb_end - kb_begin;
      if (first < gemm_units && kbs > 0) {
        ptx::fence_proxy_async_shared();  // the inits above before the loads' complete_tx
        tile_coord const c = locate(sched, first);
        pre_issued = kbs < static_cast<std::int32_t>(n_stages) ? static_cast<std::uint32_t>(kbs)
                                                               : n_stages;
        for (std::uint32_t s = 0; s < pre_issued; ++s) {
          std::int32_t const kk = (kb_begin + static_cast<std::int32_t>(s)) * kBlockK;
          std::uint8_t *sa = stages + s * stage_bytes;
          ptx::mbar_arrive_expect_tx(&full[s], tx_bytes);
          ptx::tma_load_2d(&map_a, &full[s], sa, kk, c.tile_row * kBlockM);
#pragma unroll
          for (int panel = 0; panel < BN / 64; ++panel) {
            ptx::tma_load_2d(&map_b, &full[s], sa + a_bytes + panel * cfg::b_panel_bytes,
                             c.tile_col * BN + panel * 64, kk);
          }
        }
      }
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
  if (kPair || k_split > 1) {
    ptx::cluster_sync();  // every CTA's barriers are initialised before any remote arrive
  }
  ptx::tc_fence_after_sync();
  std::uint32_t const tmem_base = *tmem_slot;
  std::uint32_t const epoch = *epoch_slot;
  std::uint32_t const parity = epoch & 1u;
  std::uint32_t *const my_events = detail::event_words(p.events);

  if constexpr (kGather) {
    // This PE's shard (written by earlier work in stream order) is readable:
    // tell every peer, before any worker of this CTA starts copying.
    if (blockIdx.x == 0 && warp == kReduceWarp0) {
      ptx::fence_acq_rel_sys();
      std::int32_t const pe = static_cast<std::int32_t>(lane);
      if (pe < p.n_pes && pe != p.my_pe) {
        ptx::st_relaxed_sys(p.peers.translate(my_events, pe) + gw.ready(p.my_pe), epoch);
      }
      __syncwarp();
    }
  }

  if (warp == 0) {
    // ---------------- task fetcher + TMA producer ----------------
    if (lane == 0) {
      // Past the loads issued during the set-up (pre_issued <= n_stages).
      std::uint32_t it = pre_issued;
      std::uint32_t stage = pre_issued == n_stages ? 0u : pre_issued;  // it % n_stages
      std::uint32_t phase = pre_issued == n_stages ? 1u : 0u;          // (it / n_stages) & 1
      bool ok = true;
      for (std::uint32_t n = 0; ok; ++n) {
        std::uint32_t const slot = n % kTaskRing;
        std::int32_t q = -1;
        if (leader) {
          // Fetch the next GEMM ticket into this CTA's ring (and the
          // follower's) once every consumer has taken the slot's last one.
          if (!bar_wait<kPair>(&task_empty[slot], ((n / kTaskRing) & 1u) ^ 1u, abort_word,
                               pipe_timeout)) {
            detail::record_error(p, err_local_timeout, 0, 0, 1);
            break;
          }
          if (k_split > 1) {
            // K split: cluster c computes tile c, once (the host launches a
            // cluster for every tile).
            std::int32_t const cluster = static_cast<std::int32_t>(blockIdx.x) / k_split;
            q = (n == 0 && cluster < gemm_units) ? cluster : -1;
          } else {
            // The first ticket of a CTA (of a pair) is its index in the grid;
            // later ones come from the queue, past those (one global atomic
            // less before the first load).
            std::uint32_t const units_in_grid = gridDim.x / (kPair ? 2u : 1u);
            std::uint32_t const ticket = n == 0 ? blockIdx.x / (kPair ? 2u : 1u)
                                                : units_in_grid + atomicAdd(&ctrl->gemm_ticket, 1u);
            q = ticket < static_cast<std::uint32_t>(gemm_units) ? static_cast<std::int32_t>(ticket)
                                                                : -1;
          }
          ring[slot] = q;
          if constexpr (kPair) {
            ptx::st_shared_remote(ptx::map_to_rank(const_cast<std::int32_t *>(&ring[slot]), 1), q);
            ptx::mbar_arrive_remote(ptx::map_to_rank(&task_full[slot], 1));
          }
          ptx::mbar_arrive(&task_full[slot]);
        } else {
          // Follower: take the ticket the leader wrote into this CTA's ring.
          if (!bar_wait<kPair>(&task_full[slot], (n / kTaskRing) & 1u, abort_word, pipe_timeout)) {
            detail::record_error(p, err_local_timeout, 0, 1, 1);
            break;
          }
          q = ring[slot];
          ptx::mbar_arrive_remote(ptx::map_to_rank(&task_empty[slot], 0));
        }
        if (q < 0) {
          break;
        }
        std::int32_t const r = tile_of(q);
        tile_coord const c = locate(sched, r);
        // SwiGLU: gate and up columns [tile_col * BN/2, + BN/2) (the leader
        // of a pair stages gate, the follower up); else B columns
        // [tile_col * BN, + BN), split between the CTAs of a pair.
        std::int32_t const b_col0 =
            kSwiGLU ? c.tile_col * (BN / 2)
                    : c.tile_col * BN + static_cast<std::int32_t>(cta_rank) * cfg::b_cols;
        CUtensorMap const *pair_b = (kSwiGLU && cta_rank == 1) ? &map_b2 : &map_b;
        // A rows: this tile's rows of A, or (all-gather) of this PE's shard
        // or of the gathered A once their tile row is copied.
        CUtensorMap const *amap = &map_a;
        std::int32_t a_row = c.tile_row * kBlockM;
        if constexpr (kGather) {
          if (c.owner == p.my_pe) {
            a_row -= p.my_pe * p.rows_per_pe;
          } else {
            amap = &map_b2;
          }
          if constexpr (kCheckBounds) {
            bool const own = c.owner == p.my_pe;
            std::int64_t const rows = own ? p.rows_per_pe : p.m;
            std::int32_t const rb = c.tile_row - c.owner * gw.mq;
            if (a_row < 0 || a_row + kBlockM > rows || c.owner < 0 || c.owner >= p.n_pes ||
                rb < 0 || rb >= gw.mq) {
              detail::record_error(p, err_bounds, static_cast<std::uint32_t>(r),
                                   static_cast<std::uint32_t>(c.owner), 31);
              break;
            }
          }
          if (c.owner != p.my_pe) {
            std::uint32_t const *rows_copied =
                my_events + gw.rows(c.owner, c.tile_row - c.owner * gw.mq);
            if (!detail::wait_at_least(rows_copied, static_cast<std::uint32_t>(p.chunks_per_block),
                                       abort_word, p.timeout_ns + kLocalTimeoutNs)) {
              detail::record_error(p, err_remote_timeout, static_cast<std::uint32_t>(r),
                                   static_cast<std::uint32_t>(c.owner), 23);
              break;
            }
            ptx::fence_proxy_async_global();  // the TMA loads read what the acquire made visible
            if (cta_rank == 0) detail::count(p, ctr_partial_acquire, kPair ? 2 : 1);
          }
        }
        std::int32_t const kb_first =
            kb_begin + (n == 0 ? static_cast<std::int32_t>(pre_issued) : 0);
        for (std::int32_t kb = kb_first; kb < kb_end; ++kb, ++it) {
          std::uint32_t const s = stage;
          if (!bar_wait<kPair>(&empty[s], phase ^ 1u, abort_word,
                               pipe_timeout)) {
            detail::record_error(p, err_local_timeout, r, 0, 2);
            ok = false;
            break;
          }
          std::uint8_t *sa = stages + s * stage_bytes;
          std::uint8_t *sb = sa + a_bytes;
          if constexpr (kPair) {
            // The pair MMAs that freed this stage read the follower's copy
            // too: pass the event on (from the second use of the stage on).
            // Relaxed: the event orders async-proxy work only (MMA reads
            // complete, then the follower's TMA overwrites), and the arrive
            // follows this thread's acquire of the MMA's commit.
            if (leader && it >= n_stages) {
              ptx::mbar_arrive_remote_relaxed(ptx::map_to_rank(&empty[s], 1));
            }
            std::uint32_t const bar = ptx::map_to_rank(&full[s], 0);
            if (leader) ptx::mbar_arrive_expect_tx(&full[s], tx_bytes);
            ptx::tma_load_2d_pair(amap, bar, sa, kb * kBlockK, a_row);
#pragma unroll
            for (int panel = 0; panel < cfg::b_cols / 64; ++panel) {
              ptx::tma_load_2d_pair(pair_b, bar, sb + panel * cfg::b_panel_bytes,
                                    b_col0 + panel * 64, kb * kBlockK);
            }
          } else {
            ptx::mbar_arrive_expect_tx(&full[s], tx_bytes);
            ptx::tma_load_2d(amap, &full[s], sa, kb * kBlockK, a_row);
#pragma unroll
            for (int panel = 0; panel < BN / 64; ++panel) {
              constexpr int kHalf = BN / 128;  // panels per half (SwiGLU)
              CUtensorMap const *map = (kSwiGLU && panel >= kHalf) ? &map_b2 : &map_b;
              std::int32_t const col = kSwiGLU ? b_col0 + (panel % kHalf) * 64 : b_col0 + panel * 64;
              ptx::tma_load_2d(map, &full[s], sb + panel * cfg::b_panel_bytes, col,
                               kb * kBlockK);
            }
          }
          if (++stage == n_stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: the most recent load of every stage must have landed before
      // this CTA may exit (normally they were all consumed already). A
      // follower's loads complete on the leader's barriers; the leader's
      // drain covers them, and the follower cannot exit before the leader
      // reaches the closing cluster barrier.
      for (std::uint32_t back = 1; leader && back <= n_stages && back <= it; ++back) {
        std::uint32_t const i = it - back;
        bar_wait<kPair>(&full[i % n_stages], (i / n_stages) & 1u, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- tcgen05.mma issuer ----------------
    // (Pairs: the leader issues for both CTAs; the follower's warp 1 only
    // holds its half of the TMEM allocation.)
    if (lane == 0 && leader) {
      std::uint32_t const idesc = ptx::idesc_bf16_f32(kPair ? 2 * kBlockM : kBlockM, BN, true);
      std::uint32_t stage = 0, phase = 0;  // position in the stage ring
      for (std::uint32_t n = 0;; ++n) {
        std::uint32_t const slot = n % kTaskRing;
        if (!ptx::mbar_wait(&task_full[slot], (n / kTaskRing) & 1u, abort_word, pipe_timeout)) {
          detail::record_error(p, err_local_timeout, 0, 0, 3);
          break;
        }
        std::int32_t const r = ring[slot];
        ptx::mbar_arrive(&task_empty[slot]);
        if (r < 0) {
          break;
        }
        std::uint32_t const buf = n & 1u;
        if (!bar_wait<kPair>(&acc_empty[buf], ((n >> 1) & 1u) ^ 1u, abort_word, pipe_timeout)) {
          detail::record_error(p, err_local_timeout, r, 0, 4);
          break;
        }
        ptx::tc_fence_after_sync();
        std::uint32_t const d_tmem = tmem_base + buf * BN;
        bool ok = true;
        for (std::int32_t kb = kb_begin; kb < kb_end; ++kb) {
          std::uint32_t const s = stage;
          if (!bar_wait<kPair>(&full[s], phase, abort_word, pipe_timeout)) {
            detail::record_error(p, err_local_timeout, r, 0, 5);
            ok = false;
            break;
          }
          ptx::tc_fence_after_sync();
          std::uint32_t const a_addr = ptx::smem_addr(stages + s * stage_bytes);
          std::uint32_t const b_addr = a_addr + a_bytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            // A: K-major, 128 B swizzle, 8-row groups 1024 B apart; a K step
            // of 16 elements is 32 B along the swizzled row.
            std::uint64_t const a_desc = ptx::smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            // B: MN-major, 128 B swizzle; 64-column panels `b_panel_bytes`
            // apart (leading), 8-k-row groups 1024 B apart (stride); a K step
            // of 16 rows is 2048 B. (Pairs: both descriptors address the
            // same offsets in both CTAs; each CTA holds its half of B.)
            std::uint64_t const b_desc =
                ptx::smem_desc_sw128(b_addr + kk * 2048, cfg::b_panel_bytes, 1024);
            std::uint32_t const acc = (kb > kb_begin || kk > 0) ? 1u : 0u;
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
          if (++stage == n_stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) {
          break;
        }
        if constexpr (kPair) {
          ptx::umma_commit_pair(&acc_full[buf]);
        } else {
          ptx::umma_commit(&acc_full[buf]);
        }
      }
      // Every issued MMA must be complete before TMEM is released.
      if constexpr (kPair) {
        ptx::umma_commit_pair(mma_done);
      } else {
        ptx::umma_commit(mma_done);
      }
      ptx::mbar_wait(mma_done, 0, nullptr, kLocalTimeoutNs);
    }
    __syncwarp();
  } else if (warp < kReduceWarp0) {
    // ---------------- epilogue: TMEM -> destination, publish ----------------
    std::int32_t const quarter = warp % 4;  // TMEM lanes [32q, 32q+32)
    std::int32_t const row_in_tile = quarter * 32 + static_cast<std::int32_t>(lane);
    for (std::uint32_t n = 0;; ++n) {
      std::uint32_t const slot = n % kTaskRing;
      // Warp-uniform decision: every lane waits, the warp acts on the vote.
      if (!__all_sync(0xffffffffu,
                      bar_wait<kPair>(&task_full[slot], (n / kTaskRing) & 1u, abort_word,
                                      pipe_timeout))) {
        if (lane == 0) detail::record_error(p, err_local_timeout, 0, cta_rank, 6);
        break;
      }
      std::int32_t const q = __shfl_sync(0xffffffffu, ring[slot], 0);
      if (lane == 0) {
        if (leader) {
          ptx::mbar_arrive(&task_empty[slot]);
        } else {
          ptx::mbar_arrive_remote(ptx::map_to_rank(&task_empty[slot], 0));
        }
      }
      if (q < 0) {
        break;
      }
      std::int32_t const r = tile_of(q);
      std::uint32_t const buf = n & 1u;
      if (!__all_sync(0xffffffffu,
                      bar_wait<kPair>(&acc_full[buf], (n >> 1) & 1u, abort_word, pipe_timeout))) {
        if (lane == 0) detail::record_error(p, err_local_timeout, r, cta_rank, 7);
        break;
      }
      if constexpr (kPair) {
        // The pair MMAs also wrote the follower's accumulator rows.
        if (leader && warp == kEpilogueWarp0 && lane == 0) {
          ptx::mbar_arrive_remote(ptx::map_to_rank(&acc_full[buf], 1));
        }
      }
      ptx::tc_fence_after_sync();
      std::uint64_t const t0 = ptx::now_ns();
      tile_coord const c = locate(sched, r);
      std::int32_t const tile = c.tile_row * p.n_tiles + c.tile_col;
      std::int32_t const grow = c.tile_row * kBlockM + row_in_tile;
      std::int32_t const gcol0 = c.tile_col * BN;
      std::uint32_t const t_row = tmem_base + (static_cast<std::uint32_t>(quarter * 32) << 16) +
                                  buf * BN;
      // Who reduces this tile: its owner (two-shot / RS) or every PE (one-shot).
      std::int32_t const first_dst = p.one_shot ? 0 : c.owner;
      std::int32_t const n_dst = p.n_pes == 1 ? 0 : (p.one_shot ? p.n_pes : 1);
      char *const slot_base = p.workspace + detail::slot_offset(parity, tile, p.tiles, kSlotBytes);
      // A 32-row quarter wholly below m carries no data: it is neither
      // written nor published, and no reduce task exists for it.
      bool const active = c.tile_row * kBlockM + quarter * 32 < p.m;

      // K split: ranks > 0 send their accumulator rows into rank 0's stage
      // ring (free once rank 0's MMAs are done); rank 0 adds them below, in
      // rank order. Layout, fp32: [rank - 1][quarter < n_active][32-column
      // chunk][4-column group][row][4 columns], so a warp's 16-byte accesses
      // cover 512 contiguous bytes on both sides.
      std::int32_t const rows_here = p.m - c.tile_row * kBlockM;
      std::int32_t const n_active = ((rows_here < kBlockM ? rows_here : kBlockM) + 31) / 32;
      float *const recv = reinterpret_cast<float *>(stages);
      if (k_split > 1) {
        if (split_rank != 0) {
          if (!__all_sync(0xffffffffu,
                          ptx::mbar_wait_cluster(ring_free, n & 1u, abort_word, pipe_timeout))) {
            if (lane == 0) detail::record_error(p, err_local_timeout, r, split_rank, 32);
            break;
          }
#pragma unroll 1
          for (int ch = 0; active && ch < BN / 32; ++ch) {
            std::uint32_t v[32];
            ptx::tmem_load_32x32b_x32(t_row + ch * 32, v);
            ptx::tmem_wait_load();
            std::uint32_t const dst = ptx::map_to_rank(
                recv + ((((static_cast<std::int32_t>(split_rank) - 1) * n_active + quarter) *
                             (BN / 32) + ch) * 1024 + static_cast<std::int32_t>(lane) * 4),
                0);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              ptx::st_shared_remote_v4(dst + j4 * 512, v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2],
                                       v[4 * j4 + 3]);
            }
          }
          ptx::tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            ptx::mbar_arrive_remote(ptx::map_to_rank(recv_full, 0));  // release: the rows above
            ptx::mbar_arrive(&acc_empty[buf]);
          }
          continue;
        }
        if (warp == kEpilogueWarp0 && lane == 0) {
          for (std::int32_t rk = 1; rk < k_split; ++rk) {
            ptx::mbar_arrive_remote(ptx::map_to_rank(ring_free, static_cast<std::uint32_t>(rk)));
          }
        }
        if (!__all_sync(0xffffffffu,
                        ptx::mbar_wait_cluster(recv_full, n & 1u, abort_word, pipe_timeout))) {
          if (lane == 0) detail::record_error(p, err_local_timeout, r, 0, 33);
          break;
        }
      }

      if constexpr (kSwiGLU) {
        // act[row, col] = silu(gate) * up, from accumulator columns col and
        // BN/2 + col, in fp32, rounded once to bf16.
        std::int32_t const acol0 = c.tile_col * (BN / 2);
#pragma unroll 1
        for (int ch = 0; active && ch < BN / 64; ++ch) {
          std::uint32_t g[32], u[32];
          ptx::tmem_load_32x32b_x32(t_row + ch * 32, g);
          ptx::tmem_load_32x32b_x32(t_row + BN / 2 + ch * 32, u);
          ptx::tmem_wait_load();
          if (grow < p.m) {
            __nv_bfloat16 *dst = p.out + static_cast<std::int64_t>(grow) * p.n;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              std::int32_t const col = acol0 + ch * 32 + j * 8;
              if (col < p.n) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  float const x = __uint_as_float(g[8 * j + e]);
                  f[e] = x / (1.0f + __expf(-x)) * __uint_as_float(u[8 * j + e]);
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
      }
#pragma unroll 1
      for (int ch = 0; !kSwiGLU && active && ch < BN / 32; ++ch) {
        std::uint32_t v[32];
        ptx::tmem_load_32x32b_x32(t_row + ch * 32, v);
        ptx::tmem_wait_load();
        for (std::int32_t rk = 1; rk < k_split; ++rk) {
          float4 const *src = reinterpret_cast<float4 const *>(
              recv + (((rk - 1) * n_active + quarter) * (BN / 32) + ch) * 1024 +
              static_cast<std::int32_t>(lane) * 4);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            float4 const f = src[j4 * 32];
            v[4 * j4 + 0] = __float_as_uint(__uint_as_float(v[4 * j4 + 0]) + f.x);
            v[4 * j4 + 1] = __float_as_uint(__uint_as_float(v[4 * j4 + 1]) + f.y);
            v[4 * j4 + 2] = __float_as_uint(__uint_as_float(v[4 * j4 + 2]) + f.z);
            v[4 * j4 + 3] = __float_as_uint(__uint_as_float(v[4 * j4 + 3]) + f.w);
          }
        }
        if (kGather || p.n_pes == 1) {
          if (grow < p.m) {
            __nv_bfloat16 *dst = p.out + static_cast<std::int64_t>(grow) * p.n;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              std::int32_t const col = gcol0 + ch * 32 + j * 8;
              if (col < p.n) {
                uint4 q;
                q.x = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 0]), __uint_as_float(v[8 * j + 1]));
                q.y = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
                q.z = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
                q.w = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
                ptx::st_v4(dst + col, q);
              }
            }
          }
        } else {
          // This PE's own partial slot (local memory); reducers read it over NVLink.
          constexpr int kVecs = 32 / kVecCols;  // wire vectors per 32-column chunk
#pragma unroll
          for (int j = 0; j < kVecs; ++j) {
            uint4 q;
            if constexpr (kWireF32) {
              q = make_uint4(v[4 * j + 0], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            } else {
              q.x = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 0]), __uint_as_float(v[8 * j + 1]));
              q.y = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
              q.z = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
              q.w = ptx::pack_bf16x2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
            }
            std::int64_t const vec = ch * kVecs + j;
            ptx::st_v4(slot_base + (vec * kBlockM + row_in_tile) * 16, q);
          }
        }
      }
      // TMEM buffer is free for the next tile once every lane has read it.
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
        detail::count(p, ctr_gemm_tasks, 1);
        detail::trace(p, 0, 0, static_cast<std::uint32_t>(r), tile, t0);
      }
      if (!active) {
        continue;
      }
      // Publish this quarter (task 0 "after" hook). The data is in this PE's
      // own memory (its out, or its partial slot that reducers load over
      // NVLink), so a GPU-scope fence suffices.
      ptx::fence_acq_rel_gpu();
      __syncwarp();
      if (kGather || p.n_pes == 1) {
        // One PE (or all-gather): the tile is final as written; mark its
        // quarter arrived.
        if (lane == 0) {
          ptx::publish_local_data(my_events + arrive_index(parity, 0, tile, quarter, 1, p.tiles),
                                  epoch);
        }
      } else if (static_cast<std::int32_t>(lane) < n_dst) {
        std::int32_t const pe = first_dst + static_cast<std::int32_t>(lane);
        std::uint32_t *flags = p.peers.translate(my_events, pe);
        ptx::publish_local_data(
            flags + arrive_index(parity, p.my_pe, tile, quarter, p.n_pes, p.tiles), epoch);
      }
      if (lane == 0) {
        detail::count(p, ctr_partial_publish, (kGather || p.n_pes == 1) ? 1 : n_dst);
      }
    }
  }

  // ---------------- workers: reduce (task 2) ----------------
  // Worker warps start at once; with comm_warps > 4 epilogue warps join once
  // the GEMM queue is drained, so the last GEMM wave's reductions use both.
  // `comm_warps` bounds how many requests a CTA keeps in flight over NVLink:
  // more only deepen the fabric's queues once it is saturated.
  int const first_comm_warp = kThreads / 32 - p.comm_warps;
  if constexpr (kGather) {
    if (warp >= first_comm_warp) {
      detail::gather_tasks(p, epoch, my_events, gw, abort_word, lane);
      if (blockIdx.x == 0 && warp == first_comm_warp) {
        detail::wait_all_reads(p, epoch, my_events, gw, abort_word, lane);
      }
    }
  } else if constexpr (!kSwiGLU) {  // the SwiGLU variant runs on one PE: no exchange
    if (p.n_pes > 1 && warp >= first_comm_warp) {
      int const worker = warp - kEpilogueWarp0;  // 0..7
      std::uint8_t *xpose = reduce_smem + worker * (32 * 128);
      if constexpr (!kWireF32) {
        if (p.mc_workspace != nullptr) {
          detail::comm_tasks_switch<BN>(p, sched, parity, epoch, my_events, abort_word, xpose,
                                        lane);
        } else if (p.comm_slices) {
          detail::comm_tasks_slices<BN>(p, sched, parity, epoch, my_events, abort_word, lane);
        } else {
          detail::comm_tasks_peer<BN, false>(p, sched, parity, epoch, my_events, abort_word,
                                             xpose, lane);
        }
      } else {
        detail::comm_tasks_peer<BN, true>(p, sched, parity, epoch, my_events, abort_word, xpose,
                                          lane);
      }
      if (p.mode == mode_allreduce && !p.one_shot) {
        detail::finish_pushes(p, parity, epoch, my_events, lane);
        if (blockIdx.x == 0 && warp == first_comm_warp) {
          detail::wait_all_pushes(p, parity, epoch, my_events, abort_word, lane);
        }
      }
    }
  }

  // ---------------- teardown ----------------
  __syncwarp();
  ptx::tc_fence_before_sync();
  __syncthreads();
  if (kPair || k_split > 1) {
    // No remote arrive, store, MMA or TMA write may still target another CTA.
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
      // Last CTA of this launch: rewind the queues and advance the epoch.
      __threadfence();
      ctrl->gemm_ticket = 0;
      ctrl->reduce_ticket = 0;
      ctrl->workers_done = 0;
      ctrl->trace_count = 0;
      if constexpr (kGather) {
        std::int64_t const first = gw.counters_first();
        for (std::int64_t i = 0; i < gw.counters_count(); ++i) my_events[first + i] = 0;
      }
      ctrl->launch_count = epoch;
      atomicAdd(&ctrl->counters[ctr_launches], 1ull);
      // No fence: nothing of this launch reads these words again, and the
      // next launch is stream-ordered after this one.
      atomicExch(&ctrl->done_ctas, 0u);
    }
  }
}

}  // namespace megacu_b200
