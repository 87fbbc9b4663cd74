// Host-only check of the event-tensor layouts (test infrastructure): every
// word the kernels index (arrive / done flags, the all-gather words, the MLP
// chain's flags and counters) is distinct and inside the size the host
// allocates. Prints "ok" and exits 0, or names the first clash.
#include <cstdint>
#include <cstdio>
#include <vector>

#include "kernels/chain_kernel.cuh"
#include "kernels/layout.h"

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

}  // namespace

int main() {
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
