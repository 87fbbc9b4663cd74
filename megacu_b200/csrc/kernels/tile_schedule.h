// Tile schedule of the fused GEMM + allreduce / reduce-scatter megakernel.
//
// The output [m, n] is cut into tile_m x tile_n tiles, tile id
// t = tile_row * n_tiles + tile_col (megacu's decomposition,
// megacu_gemm_allreduce_phased.cu:64-80). Tiles are handed out in "raster
// order": raster index r = 0, 1, ... is what the device task queue hands to
// the next free CTA. The raster order walks bands of `group_m` tile rows
// column by column, so the CTAs working at the same time share A row panels
// and B column panels in L2.
//
// Ownership (who reduces a tile) rotates with the raster index, r % n_pes,
// so every PE receives reducible tiles from the start of the GEMM. For
// reduce-scatter the owner is fixed by the output rows instead: PE q owns
// tile rows [q * mq, (q + 1) * mq); raster index r then walks PE (r % n_pes)'s
// block, so ownership still rotates in time.
//
// All-gather + GEMM (mode_allgather) has no owner: every PE computes every
// tile of its own output columns, and the rows of A arrive shard by shard
// (PE q's shard is the tile rows [q * mq, (q + 1) * mq)). The raster walks
// whole shards in the order their rows become available on this PE: its own
// shard first (`first_shard`), then the next PEs' in turn, each shard in the
// grouped order; `owner` is the shard the tile's A rows come from.
//
// The same arithmetic is restated in C in oracle/oracle.c (oracle_locate,
// oracle_locate_gather).
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define MEGACU_B200_HD __host__ __device__ __forceinline__
#else
#define MEGACU_B200_HD inline
#endif

namespace megacu_b200 {

enum : std::int32_t { mode_allreduce = 0, mode_reduce_scatter = 1, mode_allgather = 2 };

struct tile_schedule {
  std::int32_t m_tiles = 0;
  std::int32_t n_tiles = 0;
  std::int32_t n_pes = 1;
  std::int32_t mode = mode_allreduce;
  std::int32_t group_m = 16;
  std::int32_t first_shard = 0;  // mode_allgather: this PE (its shard comes first)

  MEGACU_B200_HD std::int32_t tiles() const { return m_tiles * n_tiles; }
};

struct tile_coord {
  std::int32_t tile_row = 0;
  std::int32_t tile_col = 0;
  std::int32_t owner = 0;  // PE that reduces this tile (two-shot / RS); all-gather:
                           // the PE whose shard holds the tile's A rows
  std::int32_t local = 0;  // index of this tile among its owner's tiles
};

// Grouped raster walk of an (rows x cols) tile grid: r -> (row, col).
MEGACU_B200_HD void grouped_raster(std::int32_t r, std::int32_t rows, std::int32_t cols,
                                   std::int32_t group, std::int32_t &row,
                                   std::int32_t &col) {
  std::int32_t const band_tiles = group * cols;
  std::int32_t const band = r / band_tiles;
  std::int32_t const first_row = band * group;
  std::int32_t const left = rows - first_row;
  std::int32_t const band_rows = left < group ? left : group;
  std::int32_t const within = r - band * band_tiles;
  row = first_row + within % band_rows;
  col = within / band_rows;
}

MEGACU_B200_HD tile_coord locate(tile_schedule const &s, std::int32_t r) {
  tile_coord c;
  if (s.mode == mode_allgather) {
    std::int32_t const mq = s.m_tiles / s.n_pes;
    std::int32_t const per_shard = mq * s.n_tiles;
    std::int32_t const d = r / per_shard;
    c.local = r - d * per_shard;
    c.owner = (s.first_shard + d) % s.n_pes;
    std::int32_t row = 0;
    grouped_raster(c.local, mq, s.n_tiles, s.group_m < mq ? s.group_m : mq, row, c.tile_col);
    c.tile_row = c.owner * mq + row;
    return c;
  }
  c.owner = r % s.n_pes;
  c.local = r / s.n_pes;
  if (s.mode == mode_reduce_scatter) {
    std::int32_t const mq = s.m_tiles / s.n_pes;
    std::int32_t row = 0;
    grouped_raster(c.local, mq, s.n_tiles, s.group_m < mq ? s.group_m : mq, row,
                   c.tile_col);
    c.tile_row = c.owner * mq + row;
  } else {
    grouped_raster(r, s.m_tiles, s.n_tiles, s.group_m, c.tile_row, c.tile_col);
  }
  return c;
}

// CTA-pair schedule. The two CTAs of a cluster compute the two vertically
// adjacent 128-row tiles (2i, col) and (2i + 1, col) of one 256-row pair
// tile; the GEMM queue then hands out pair tickets q, and CTA `rank` (0 or 1)
// of the pair computes raster index pair_raster(q, rank). Allreduce: the
// raster walks a band's rows column by column, so with an even band height
// r = 2q and 2q + 1 are such neighbours. Reduce-scatter: PE o's tiles have
// raster indices local * n_pes + o, and locals 2u, 2u + 1 are neighbours in
// o's row block. All-gather: a shard's tiles are walked like an allreduce
// raster of its mq tile rows, so with mq and the band height even, r = 2q
// and 2q + 1 are again neighbours (and in the same shard).
MEGACU_B200_HD bool pairs_fit(tile_schedule const &s) {
  if (s.group_m % 2 != 0) {
    return false;
  }
  if (s.mode == mode_reduce_scatter || s.mode == mode_allgather) {
    return (s.m_tiles / s.n_pes) % 2 == 0;
  }
  return s.m_tiles % 2 == 0;
}

MEGACU_B200_HD std::int32_t pair_raster(tile_schedule const &s, std::int32_t q,
                                        std::int32_t rank) {
  if (s.mode == mode_reduce_scatter) {
    return (2 * (q / s.n_pes) + rank) * s.n_pes + q % s.n_pes;
  }
  return 2 * q + rank;
}

// All-gather copy chunk: whole rows of A, about 64 KiB (a power of two of
// rows, so that a 128-row tile row is a whole number of chunks).
MEGACU_B200_HD std::int32_t gather_chunk_rows(std::int64_t k) {
  std::int32_t rows = 128;
  while (rows > 1 && static_cast<std::int64_t>(rows) * k * 2 > 65536) rows /= 2;
  return rows;
}

// All-gather copy ticket t of PE my_pe -> the chunk it copies. Tickets walk
// shard slots (slot s = the shard of the PE s + 1 hops away; the last slot
// this PE's own shard), then tile rows of the shard, then chunks of
// chunk_rows rows within the tile row (chunks_per_block of them).
struct gather_chunk {
  std::int32_t hops = 0;  // PEs away from my_pe (0: this PE's own shard)
  std::int32_t src = 0;   // PE whose shard the chunk belongs to
  std::int32_t rb = 0;    // tile row within the shard
  std::int32_t row0 = 0;  // first row of the chunk within the shard
};

MEGACU_B200_HD gather_chunk locate_gather_chunk(std::int32_t ticket, std::int32_t n_pes,
                                                std::int32_t my_pe, std::int32_t mq,
                                                std::int32_t chunks_per_block,
                                                std::int32_t chunk_rows) {
  std::int32_t const per_shard = mq * chunks_per_block;
  std::int32_t const slot = ticket / per_shard;
  std::int32_t const within = ticket - slot * per_shard;
  gather_chunk g;
  g.rb = within / chunks_per_block;
  g.hops = (slot + 1) % n_pes;
  g.src = (my_pe + g.hops) % n_pes;
  g.row0 = g.rb * 128 + (within - g.rb * chunks_per_block) * chunk_rows;
  return g;
}

// Number of tiles PE q reduces under the two-shot / reduce-scatter split.
MEGACU_B200_HD std::int32_t owned_tiles(tile_schedule const &s, std::int32_t q) {
  std::int32_t const t = s.tiles();
  return t > q ? (t - q + s.n_pes - 1) / s.n_pes : 0;
}

}  // namespace megacu_b200

#undef MEGACU_B200_HD
