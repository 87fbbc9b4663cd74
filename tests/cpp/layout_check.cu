// Host-only check of the event-tensor layouts (test infrastructure): every
// word the kernels index (arrive / done flags, the all-gather words, the MLP
// chain's flags and counters) is distinct and inside the size the host
// allocates. Prints "ok" and exits 0, or names the first clash.
#include <cstdint>
#include <cstdio>
#include <vector>

#include "kernels/chain_kernel.cuh"
#include "kernels/layout.h"
#include "kernels/tile_schedule.h"

using namespace megacu_b200;

namespace {

bool claim(std::vector<int> &used, std::int64_t word, char const *what) {
  if (word < 0 || word >= static_cast<std::int64_t>(used.size())) {
    std::printf("%s: word %lld outside %zu\n", what, static_cast<long long>(word), used.size());
    return false;
  }
  if (used[word]++) {
    std::printf("%s: word %lld used twice\n", what, static_cast<long long>(word));
    return false;
  }
  return true;
}

bool check_gemm_ar(int n_pes, int tiles) {
  std::vector<int> used((events_bytes_for(n_pes, tiles) - kControlBytes) / 4, 0);
  for (int p = 0; p < 2; ++p)
    for (int src = 0; src < n_pes; ++src)
      for (int t = 0; t < tiles; ++t)
        for (int q = 0; q < kQuarters; ++q)
          if (!claim(used, arrive_index(p, src, t, q, n_pes, tiles), "arrive")) return false;
  for (int p = 0; p < 2; ++p)
    for (int src = 0; src < n_pes; ++src)
      if (!claim(used, done_index(p, src, n_pes, tiles), "done")) return false;
  return true;
}

bool check_gather(int n_pes, int tiles, int mq) {
  std::vector<int> used((events_bytes_for_gather(n_pes, tiles, mq) - kControlBytes) / 4, 0);
  gather_words const gw = gather_layout(n_pes, tiles, mq);
  for (int p = 0; p < 2; ++p)
    for (int t = 0; t < tiles; ++t)
      for (int q = 0; q < kQuarters; ++q)
        if (!claim(used, arrive_index(p, 0, t, q, 1, tiles), "gather arrive")) return false;
  for (int s = 0; s < n_pes; ++s) {
    if (!claim(used, gw.ready(s), "ready") || !claim(used, gw.read_done(s), "read_done") ||
        !claim(used, gw.chunks(s), "chunks"))
      return false;
    for (int rb = 0; rb < mq; ++rb)
      if (!claim(used, gw.rows(s, rb), "rows")) return false;
  }
  if (gw.counters_first() + gw.counters_count() != gw.end()) {
    std::printf("gather counters do not end the region\n");
    return false;
  }
  return true;
}

bool check_chain(int layers, int n_pes, int m_tiles, int dn_tiles_n) {
  std::vector<int> used((chain_events_bytes(layers, n_pes, dn_tiles_n, m_tiles) - kControlBytes) / 4,
                        0);
  for (int l = 0; l < layers; ++l)
    for (int src = 0; src < n_pes; ++src)
      for (int t = 0; t < m_tiles * dn_tiles_n; ++t)
        for (int q = 0; q < 4; ++q)
          if (!claim(used, chain_arrive_index(l, src, t, q, n_pes, dn_tiles_n, m_tiles),
                     "chain arrive"))
            return false;
  for (int l = 0; l < layers; ++l)
    for (int row = 0; row < m_tiles; ++row)
      if (!claim(used, chain_act_ready_index(l, row, layers, n_pes, dn_tiles_n, m_tiles),
                 "act_ready") ||
          !claim(used, chain_x_ready_index(l, row, layers, n_pes, dn_tiles_n, m_tiles),
                 "x_ready"))
        return false;
  return true;
}

// The all-gather schedule of every PE: the copy tickets cover every row of
// every shard exactly once, inside its shard, own shard last; the GEMM raster
// covers every tile once, whole shards in copy order, and every A row a tile
// reads (own shard in place, others in the gathered A) and every counter it
// waits on is in range.
bool check_gather_schedule(int n_pes, int mq, int n_tiles, long long k) {
  int const rows_per_pe = mq * 128;
  int const chunk_rows = gather_chunk_rows(k);
  int const per_block = 128 / chunk_rows;
  int const tickets = n_pes * mq * per_block;
  if (128 % chunk_rows != 0 || (chunk_rows > 1 && chunk_rows * k * 2 > 65536)) {
    std::printf("chunk rows %d for k %lld\n", chunk_rows, k);
    return false;
  }
  gather_words const gw = gather_layout(n_pes, mq * n_pes * n_tiles, mq);
  for (int me = 0; me < n_pes; ++me) {
    std::vector<int> row_seen(static_cast<std::size_t>(n_pes) * rows_per_pe, 0);
    int last_hops = 1;
    for (int t = 0; t < tickets; ++t) {
      gather_chunk const c = locate_gather_chunk(t, n_pes, me, mq, per_block, chunk_rows);
      if (c.src < 0 || c.src >= n_pes || c.row0 < 0 || c.row0 + chunk_rows > rows_per_pe ||
          c.rb != c.row0 / 128 || (c.src - me + n_pes) % n_pes != c.hops) {
        std::printf("copy ticket %d of PE %d out of range\n", t, me);
        return false;
      }
      int const order = c.hops == 0 ? n_pes : c.hops;  // own shard last
      if (order < last_hops) {
        std::printf("copy ticket %d of PE %d out of order\n", t, me);
        return false;
      }
      last_hops = order;
      for (int r = 0; r < chunk_rows; ++r) row_seen[c.src * rows_per_pe + c.row0 + r] += 1;
    }
    for (std::size_t i = 0; i < row_seen.size(); ++i) {
      if (row_seen[i] != 1) {
        std::printf("gathered row %zu copied %d times on PE %d\n", i, row_seen[i], me);
        return false;
      }
    }
    tile_schedule const s{mq * n_pes, n_tiles, n_pes, mode_allgather, 16, me};
    std::vector<int> tile_seen(static_cast<std::size_t>(s.tiles()), 0);
    for (int r = 0; r < s.tiles(); ++r) {
      tile_coord const c = locate(s, r);
      int const hops = (c.owner - me + n_pes) % n_pes;
      if (hops != r / (mq * n_tiles) || c.tile_row < c.owner * mq ||
          c.tile_row >= (c.owner + 1) * mq || c.tile_col < 0 || c.tile_col >= n_tiles) {
        std::printf("raster %d of PE %d out of shard\n", r, me);
        return false;
      }
      tile_seen[c.tile_row * n_tiles + c.tile_col] += 1;
      if (c.owner == me) {
        int const a_row = c.tile_row * 128 - me * rows_per_pe;
        if (a_row < 0 || a_row + 128 > rows_per_pe) return false;
      } else {
        std::int64_t const w = gw.rows(c.owner, c.tile_row - c.owner * mq);
        if (w < gw.counters_first() || w >= gw.counters_first() + n_pes * mq) return false;
      }
    }
    for (int v : tile_seen) {
      if (v != 1) {
        std::printf("a tile computed %d times on PE %d\n", v, me);
        return false;
      }
    }
  }
  return true;
}

}  // namespace

int main() {
  for (int n_pes : {1, 2, 3, 8})
    for (int mq : {1, 2, 8})
      for (int n_tiles : {1, 5, 14})
        for (long long k : {8LL, 200LL, 4096LL, 8192LL, 65536LL})
          if (!check_gather_schedule(n_pes, mq, n_tiles, k)) return 1;
  for (int n_pes : {1, 2, 3, 8})
    for (int tiles : {1, 7, 64}) {
      if (!check_gemm_ar(n_pes, tiles)) return 1;
      for (int mq : {1, 2, 5})
        if (!check_gather(n_pes, tiles, mq)) return 1;
    }
  for (int layers : {1, 2, 6})
    for (int n_pes : {1, 2, 8})
      for (int m_tiles : {1, 3, 16})
        for (int dn : {1, 4, 16})
          if (!check_chain(layers, n_pes, m_tiles, dn)) return 1;
  std::printf("ok\n");
  return 0;
}
