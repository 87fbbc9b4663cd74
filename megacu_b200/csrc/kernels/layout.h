// Memory layout of the caller-provided `events` and `workspace` buffers of
// the bf16 megakernel.
//
// events (uint32 words, symmetric when n_pes > 1):
//   [0, 256 B)  control block: device task-queue tickets, the launch counter
//               that tags every flag with the call's epoch, the error word
//               and cumulative completion counters.
//   then the event tensor, two regions of uint32 flags:
//     arrive[p][src][t][q]  (p < 2, src < n_pes, q < 4) = epoch once PE `src`
//         has delivered rows [32q, 32q + 32) of its partial of tile t;
//     done[p][src]          (src < n_pes) = epoch once PE `src` has written
//         every block it reduced into this PE's `out` (two-shot allreduce,
//         where each owner stores its summed tiles into every PE's out).
//   This is megacu's event tensor int32 [n_pes][tiles]
//   (backends/nvshmem/cuda_event_tensor.cuh:13-39) refined to quarter tiles
//   and tagged with the epoch (the golden's ready_base idiom,
//   golden_gemm_allreduce.cu:384-385), so consecutive calls need no memset
//   and no host barrier; the parity plane lets a PE run one call ahead of a
//   slow owner in reduce-scatter mode.
//
// All-gather + GEMM (mode_allgather) uses the arrive plane of a one-PE call
// (arrive[p][0][t][q] = epoch once this PE's tile quarter is stored) and
// then, per PE, a gather region of uint32 words:
//   ready[src]       = epoch once PE `src` has announced that its A shard is
//                      readable (set by `src` at the start of its call);
//   read_done[src]   = epoch once PE `src` has copied all of this PE's shard
//                      (set by `src`; this PE's call ends only after every
//                      peer's, so the next writer of the shard cannot race
//                      a peer still reading it);
//   rows[shard][rb]  local count of copied chunks of tile row rb of `shard`
//                      (the GEMM's A operand is ready at chunks_per_block);
//   chunks[src]      local count of copied chunks of `src`'s shard.
// The two counter arrays are zeroed by the last CTA of every launch.
//
// workspace (symmetric when n_pes > 1): this PE's own partial tiles,
//   slot[p][t] = the tile_m x tile_n partial of tile t (wire dtype), written
//   by this PE's epilogue into its own memory and read over NVLink by the
//   tile's reducers. Inside a slot, 16-byte vectors are stored column-major
//   over rows: vector (v, row) at byte (v * tile_m + row) * 16, which is the
//   order the TMEM epilogue produces them in (one warp access = 512 B).
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define MEGACU_B200_LAYOUT_HD __host__ __device__
#else
#define MEGACU_B200_LAYOUT_HD
#endif

namespace megacu_b200 {

inline constexpr std::int64_t kControlBytes = 256;
inline constexpr std::int32_t kQuarters = 4;   // 32-row quarters of a 128-row tile
inline constexpr std::int32_t kColBlocks = 4;  // 64-column blocks of a tile (at most)

struct control_block {
  std::uint32_t gemm_ticket;    // next GEMM raster index to hand out
  std::uint32_t reduce_ticket;  // next reduce sub-task to hand out
  std::uint32_t done_ctas;      // CTAs finished in this launch
  std::uint32_t launch_count;   // completed launches on this buffer
  std::uint32_t error_code;     // 0 = ok; non-zero = first error seen
  std::uint32_t error_info[3];  // tile, peer, site of that error
  std::uint32_t trace_count;    // trace records written
  std::uint32_t workers_done;   // reduce workers finished in this launch
  std::uint32_t reserved[6];
  unsigned long long counters[8];
};
static_assert(sizeof(control_block) <= kControlBytes, "control block too large");

enum : std::uint32_t {
  err_none = 0,
  err_remote_timeout = 40,  // a cross-GPU flag never arrived
  err_local_timeout = 41,   // an on-chip pipeline wait timed out
  err_bounds = 42,          // a bounds check of the checked build failed
};

// The bounds-checked build (-DMEGACU_B200_DEBUG_BOUNDS, libmegacu_b200_checked.so):
// the kernels check the index of each access whose arithmetic is theirs (copy
// chunks, exchange slots and rows, event words, TMA row coordinates) against
// the extent of its buffer; a failed check records err_bounds with the site
// and skips the access instead of making it. The regular build compiles the
// checks away.
#if defined(MEGACU_B200_DEBUG_BOUNDS)
inline constexpr bool kCheckBounds = true;
#else
inline constexpr bool kCheckBounds = false;
#endif

enum : std::int32_t {
  ctr_gemm_tasks = 0,
  ctr_reduce_tasks = 1,
  ctr_partial_publish = 2,
  ctr_partial_acquire = 3,
  ctr_final_publish = 4,
  ctr_final_acquire = 5,
  ctr_launches = 6,
  ctr_errors = 7,
};

// Word index (after the control block) of arrive[p][src][t][q].
MEGACU_B200_LAYOUT_HD inline std::int64_t arrive_index(std::int32_t parity, std::int32_t src,
                                                     std::int32_t tile, std::int32_t quarter,
                                                     std::int32_t n_pes, std::int32_t tiles) {
  return ((static_cast<std::int64_t>(parity) * n_pes + src) * tiles + tile) * kQuarters + quarter;
}

// Word index (after the control block) of done[p][src].
MEGACU_B200_LAYOUT_HD inline std::int64_t done_index(std::int32_t parity, std::int32_t src,
                                                   std::int32_t n_pes, std::int32_t tiles) {
  return static_cast<std::int64_t>(2) * n_pes * tiles * kQuarters +
         static_cast<std::int64_t>(parity) * n_pes + src;
}

// Word indices (after the control block) of the all-gather region.
struct gather_words {
  std::int64_t base;     // first word of the region
  std::int32_t n_pes;
  std::int32_t mq;       // tile rows per shard

  MEGACU_B200_LAYOUT_HD std::int64_t ready(std::int32_t src) const { return base + src; }
  MEGACU_B200_LAYOUT_HD std::int64_t read_done(std::int32_t src) const {
    return base + n_pes + src;
  }
  MEGACU_B200_LAYOUT_HD std::int64_t rows(std::int32_t shard, std::int32_t rb) const {
    return base + 2 * n_pes + static_cast<std::int64_t>(shard) * mq + rb;
  }
  MEGACU_B200_LAYOUT_HD std::int64_t chunks(std::int32_t src) const {
    return base + 2 * n_pes + static_cast<std::int64_t>(n_pes) * mq + src;
  }
  // Words of the two counter arrays (rows then chunks), zeroed per launch.
  MEGACU_B200_LAYOUT_HD std::int64_t counters_first() const { return rows(0, 0); }
  MEGACU_B200_LAYOUT_HD std::int64_t counters_count() const {
    return static_cast<std::int64_t>(n_pes) * mq + n_pes;
  }
  MEGACU_B200_LAYOUT_HD std::int64_t end() const { return chunks(n_pes); }
};

MEGACU_B200_LAYOUT_HD inline gather_words gather_layout(std::int32_t n_pes, std::int32_t tiles,
                                                       std::int32_t mq) {
  return gather_words{static_cast<std::int64_t>(2) * tiles * kQuarters, n_pes, mq};
}

inline std::int64_t events_bytes_for_gather(std::int32_t n_pes, std::int32_t tiles,
                                            std::int32_t mq) {
  return kControlBytes + 4 * gather_layout(n_pes, tiles, mq).end();
}

inline std::int64_t events_bytes_for(std::int32_t n_pes, std::int32_t tiles) {
  std::int64_t const words = static_cast<std::int64_t>(2) * n_pes * tiles * kQuarters +
                             static_cast<std::int64_t>(2) * n_pes;
  return kControlBytes + 4 * words;
}

}  // namespace megacu_b200

#undef MEGACU_B200_LAYOUT_HD
