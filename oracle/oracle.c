/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle of the fused GEMM + allreduce /
 * reduce-scatter path (see oracle.h for what it restates and where each
 * part comes from in the reference). Nothing in the product links this.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- fp32 GEMM, k ascending, one fmaf per step ---------------------------
 * Restates golden/golden_gemm_allreduce.cu:85-96 and
 * megacu_gemm_allreduce_phased.cu:82-87 (`value += a * b`, which nvcc
 * contracts to a fused multiply-add). Iterating k in the outer loop of a row
 * block keeps that per-element order while streaming b rows. */
void oracle_gemm_block(const float *a, const float *b, float *c, int64_t m, int64_t n,
                       int64_t k, int64_t r0, int64_t r1, int64_t c0, int64_t c1) {
  (void)m;
  enum { kColBlock = 512, kDepthBlock = 128 };
  for (int64_t r = r0; r < r1; ++r) {
    for (int64_t j = c0; j < c1; ++j) c[r * n + j] = 0.0f;
  }
  /* Blocked over columns and k so the b panel stays in cache; every element
   * still accumulates k = 0, 1, ..., k-1 in that order. */
  for (int64_t cb = c0; cb < c1; cb += kColBlock) {
    int64_t const ce = cb + kColBlock < c1 ? cb + kColBlock : c1;
    int64_t const w = ce - cb;
    for (int64_t k0 = 0; k0 < k; k0 += kDepthBlock) {
      int64_t const k1 = k0 + kDepthBlock < k ? k0 + kDepthBlock : k;
      for (int64_t r = r0; r < r1; ++r) {
        float *crow = c + r * n + cb;
        const float *arow = a + r * k;
        for (int64_t kk = k0; kk < k1; ++kk) {
          float const av = arow[kk];
          const float *brow = b + kk * n + cb;
          for (int64_t j = 0; j < w; ++j) crow[j] = fmaf(av, brow[j], crow[j]);
        }
      }
    }
  }
}

typedef struct gemm_job {
  const float *a, *b;
  float *c;
  int64_t m, n, k, r0, r1;
} gemm_job;

static void *gemm_worker(void *arg) {
  gemm_job *j = (gemm_job *)arg;
  oracle_gemm_block(j->a, j->b, j->c, j->m, j->n, j->k, j->r0, j->r1, 0, j->n);
  return NULL;
}

void oracle_gemm_f32(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                     int32_t threads) {
  if (threads <= 1 || m < 2) {
    oracle_gemm_block(a, b, c, m, n, k, 0, m, 0, n);
    return;
  }
  if (threads > m) threads = (int32_t)m;
  pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
  gemm_job *jobs = (gemm_job *)malloc(sizeof(gemm_job) * (size_t)threads);
  for (int32_t t = 0; t < threads; ++t) {
    jobs[t].a = a;
    jobs[t].b = b;
    jobs[t].c = c;
    jobs[t].m = m;
    jobs[t].n = n;
    jobs[t].k = k;
    jobs[t].r0 = m * t / threads;
    jobs[t].r1 = m * (t + 1) / threads;
    pthread_create(&tid[t], NULL, gemm_worker, &jobs[t]);
  }
  for (int32_t t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(jobs);
  free(tid);
}

float oracle_round_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) {
    if (u & 0x007fffffu) u |= 0x00400000u; /* quiet NaN */
    u &= 0xffff0000u;
  } else {
    uint32_t const lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    u &= 0xffff0000u;
  }
  memcpy(&x, &u, 4);
  return x;
}

/* ---- megacu's phased fp32 graph -------------------------------------------- */

int oracle_phased_f32(int64_t m, int64_t n, int64_t k, int32_t tile_m, int32_t tile_n,
                      int32_t n_pes, const float *const *a, const float *const *b,
                      float *const *out, int32_t *const *events) {
  int64_t const n_tiles = (n + tile_n - 1) / tile_n;
  int64_t const tiles = ((m + tile_m - 1) / tile_m) * n_tiles;
  float **partial = (float **)calloc((size_t)n_pes, sizeof(float *));
  int rc = 0;
  for (int32_t pe = 0; pe < n_pes; ++pe) {
    memset(events[pe], 0, sizeof(int32_t) * (size_t)(tiles * n_pes));
  }
  /* Task 0 on every PE, tile by tile, then publish tile + 1 into every PE's
   * slot [pe][tile] (cuda_event_tensor.cuh:19-31). */
  for (int32_t pe = 0; pe < n_pes; ++pe) {
    partial[pe] = (float *)calloc((size_t)(m * n), sizeof(float));
    for (int64_t t = 0; t < tiles; ++t) {
      int64_t const r0 = (t / n_tiles) * tile_m, c0 = (t % n_tiles) * tile_n;
      int64_t const r1 = r0 + tile_m < m ? r0 + tile_m : m;
      int64_t const c1 = c0 + tile_n < n ? c0 + tile_n : n;
      oracle_gemm_block(a[pe], b[pe], partial[pe], m, n, k, r0, r1, c0, c1);
      for (int32_t dst = 0; dst < n_pes; ++dst) events[dst][pe * tiles + t] = (int32_t)(t + 1);
    }
  }
  /* Task 2 on every PE: acquire all slots of the tile, then sum in PE order
   * (megacu_gemm_allreduce_phased.cu:118-130). */
  for (int32_t pe = 0; pe < n_pes && rc == 0; ++pe) {
    for (int64_t t = 0; t < tiles && rc == 0; ++t) {
      for (int32_t src = 0; src < n_pes; ++src) {
        if (events[pe][src * tiles + t] != (int32_t)(t + 1)) rc = -1;
      }
      int64_t const r0 = (t / n_tiles) * tile_m, c0 = (t % n_tiles) * tile_n;
      for (int64_t r = r0; r < r0 + tile_m && r < m; ++r) {
        for (int64_t c = c0; c < c0 + tile_n && c < n; ++c) {
          float s = 0.0f;
          for (int32_t src = 0; src < n_pes; ++src) s += partial[src][r * n + c];
          out[pe][r * n + c] = s;
        }
      }
    }
  }
  for (int32_t pe = 0; pe < n_pes; ++pe) free(partial[pe]);
  free(partial);
  return rc;
}

/* ---- B200 megakernel schedule (restates tile_schedule.h) ------------------- */

static void grouped_raster(int32_t r, int32_t rows, int32_t cols, int32_t group, int32_t *row,
                           int32_t *col) {
  int32_t const band_tiles = group * cols;
  int32_t const band = r / band_tiles;
  int32_t const first = band * group;
  int32_t const left = rows - first;
  int32_t const band_rows = left < group ? left : group;
  int32_t const within = r - band * band_tiles;
  *row = first + within % band_rows;
  *col = within / band_rows;
}

void oracle_locate(int32_t m_tiles, int32_t n_tiles, int32_t n_pes, int32_t mode,
                   int32_t group_m, int32_t r, int32_t out[4]) {
  out[2] = r % n_pes;
  out[3] = r / n_pes;
  if (mode == 1) {
    int32_t const mq = m_tiles / n_pes;
    int32_t row, col;
    grouped_raster(out[3], mq, n_tiles, group_m < mq ? group_m : mq, &row, &col);
    out[0] = out[2] * mq + row;
    out[1] = col;
  } else {
    grouped_raster(r, m_tiles, n_tiles, group_m, &out[0], &out[1]);
  }
}

void oracle_pair_raster(int32_t n_pes, int32_t mode, int32_t q, int32_t out[2]) {
  for (int32_t rank = 0; rank < 2; ++rank) {
    /* allreduce: raster neighbours 2q, 2q + 1 (a band is walked column by
     * column); reduce-scatter: owner q % n_pes's local tiles 2u, 2u + 1. */
    out[rank] = mode == 1 ? (2 * (q / n_pes) + rank) * n_pes + q % n_pes : 2 * q + rank;
  }
}

/* Event tensor words after the control block (restates layout.h):
 * arrive[p][src][t][q] (q < 4 quarters), then done[p][src]. */
static int64_t arrive_idx(int32_t parity, int32_t src, int32_t tile, int32_t quarter,
                          int32_t n_pes, int32_t tiles) {
  return (((int64_t)parity * n_pes + src) * tiles + tile) * 4 + quarter;
}

static int64_t done_idx(int32_t parity, int32_t src, int32_t n_pes, int32_t tiles) {
  return (int64_t)2 * n_pes * tiles * 4 + (int64_t)parity * n_pes + src;
}

/* Does quarter q x 64-column block c of tile (row, col) hold an output element? */
static int block_exists(const oracle_bf16_problem *p, int32_t row, int32_t col, int32_t q,
                        int32_t c) {
  return (int64_t)row * p->tile_m + q * 32 < p->m && (int64_t)col * p->tile_n + c * 64 < p->n;
}

int oracle_bf16_call(const oracle_bf16_problem *p, const float *const *a,
                     const float *const *b, float *const *out, uint32_t *const *events,
                     uint64_t *counters, int32_t *gemm_order, int32_t *const *reduce_order) {
  int32_t const np = p->n_pes;
  int64_t const m = p->m, n = p->n;
  int32_t const mt = (int32_t)((m + p->tile_m - 1) / p->tile_m);
  int32_t const nt = (int32_t)((n + p->tile_n - 1) / p->tile_n);
  int32_t const tiles = mt * nt;
  uint32_t const epoch = p->epoch;
  int32_t const parity = (int32_t)(epoch & 1u);
  int const two_shot_ar = p->mode == 0 && !p->one_shot && np > 1;
  int rc = 0;
  uint64_t local_counters[8 * 8];
  uint64_t *cnt = counters != NULL ? counters : local_counters;
  memset(cnt, 0, sizeof(uint64_t) * 8 * (size_t)np);

  /* Every PE's full partial product (what its GEMM tiles produce). */
  float **part = (float **)calloc((size_t)np, sizeof(float *));
  for (int32_t pe = 0; pe < np; ++pe) {
    part[pe] = (float *)malloc(sizeof(float) * (size_t)(m * n));
    oracle_gemm_f32(a[pe], b[pe], part[pe], m, n, p->k, p->threads);
    if (np > 1 && p->wire_bytes == 2) {
      for (int64_t i = 0; i < m * n; ++i) part[pe][i] = oracle_round_bf16(part[pe][i]);
    }
  }

  int32_t const blocks = p->tile_n / 64;

  /* Task 0 (GEMM tile) + its publish, in queue (raster) order. */
  for (int32_t r = 0; r < tiles; ++r) {
    int32_t c[4];
    oracle_locate(mt, nt, np, p->mode, p->group_m, r, c);
    int32_t const t = c[0] * nt + c[1];
    if (gemm_order) gemm_order[r] = t;
    for (int32_t pe = 0; pe < np; ++pe) {
      cnt[pe * 8 + 0] += 1;
      for (int32_t q = 0; q < 4; ++q) {
        if ((int64_t)c[0] * p->tile_m + q * 32 >= m) continue;
        if (np == 1) {
          /* One PE: the quarter is arrived (the tile is final as written). */
          if (events) events[0][arrive_idx(parity, 0, t, q, 1, tiles)] = epoch;
          cnt[pe * 8 + 2] += 1;
        } else {
          int32_t const first = p->one_shot ? 0 : c[2];
          int32_t const n_dst = p->one_shot ? np : 1;
          for (int32_t d = 0; d < n_dst; ++d) {
            if (events) events[first + d][arrive_idx(parity, pe, t, q, np, tiles)] = epoch;
          }
          cnt[pe * 8 + 2] += (uint64_t)n_dst;
        }
      }
    }
  }

  if (np == 1) {
    memcpy(out[0], part[0], sizeof(float) * (size_t)(m * n));
  } else {
    int64_t const rows_per_pe = m / np;
    int32_t const per_tile = 4 * blocks;
    for (int32_t me = 0; me < np && rc == 0; ++me) {
      /* Task 2 queue: every (reduced tile, 32-row quarter, 64-column block),
       * the reduced tiles being this PE's own (two-shot, reduce-scatter) or
       * all of them (one-shot), in raster order. (The kernel's queue hands
       * out (tile, quarter) tickets and reduces their blocks in order: the
       * same sequence.) */
      int32_t const reduced = p->one_shot ? tiles : (tiles > me ? (tiles - me + np - 1) / np : 0);
      for (int32_t ticket = 0; ticket < reduced * per_tile && rc == 0; ++ticket) {
        int32_t const j = ticket / per_tile;
        int32_t const q = (ticket % per_tile) / blocks;
        int32_t const cb = ticket % blocks;
        int32_t const r = p->one_shot ? j : j * np + me;
        int32_t c[4];
        oracle_locate(mt, nt, np, p->mode, p->group_m, r, c);
        int32_t const t = c[0] * nt + c[1];
        if (!block_exists(p, c[0], c[1], q, cb)) {
          if (reduce_order) reduce_order[me][ticket] = -1;
          continue;
        }
        if (reduce_order) reduce_order[me][ticket] = t;
        /* Task 2 "before": acquire every PE's quarter. */
        if (events) {
          for (int32_t src = 0; src < np; ++src) {
            if (events[me][arrive_idx(parity, src, t, q, np, tiles)] != epoch) rc = -2;
          }
        }
        cnt[me * 8 + 1] += 1;
        cnt[me * 8 + 3] += (uint64_t)np;
        int64_t const row0 = (int64_t)c[0] * p->tile_m + q * 32;
        int64_t const c0 = (int64_t)c[1] * p->tile_n + cb * 64;
        for (int64_t row = row0; row < row0 + 32 && row < m; ++row) {
          for (int64_t col = c0; col < c0 + 64 && col < n; ++col) {
            float s = 0.0f;
            for (int32_t src = 0; src < np; ++src) s += part[src][row * n + col];
            if (p->mode == 1) {
              out[me][(row - me * rows_per_pe) * n + col] = s;
            } else if (p->one_shot) {
              out[me][row * n + col] = s;
            } else {
              for (int32_t pe = 0; pe < np; ++pe) out[pe][row * n + col] = s; /* into every out */
            }
          }
        }
        if (two_shot_ar) cnt[me * 8 + 4] += (uint64_t)np;
      }
      /* Two-shot completion: PE me announces on every PE that all of its
       * blocks are written. */
      if (two_shot_ar && events) {
        for (int32_t pe = 0; pe < np; ++pe) events[pe][done_idx(parity, me, np, tiles)] = epoch;
      }
    }
    if (two_shot_ar) {
      /* Every PE's call completes once every PE's done flag is set. */
      for (int32_t pe = 0; pe < np; ++pe) {
        for (int32_t src = 0; src < np; ++src) {
          if (events && events[pe][done_idx(parity, src, np, tiles)] != epoch) rc = -3;
        }
        cnt[pe * 8 + 5] += (uint64_t)np;
      }
    }
  }
  for (int32_t pe = 0; pe < np; ++pe) {
    cnt[pe * 8 + 6] += 1;
    free(part[pe]);
  }
  free(part);
  return rc;
}

/* ---- all-gather + GEMM (a B200 addition; restates tile_schedule.h's
 *      mode_allgather raster and layout.h's gather words) ------------------ */

void oracle_locate_gather(int32_t m_tiles, int32_t n_tiles, int32_t n_pes, int32_t my_pe,
                          int32_t group_m, int32_t r, int32_t out[4]) {
  /* Whole shards in the order their rows are present on PE my_pe: its own
   * first, then the PEs 1, 2, ... hops further; a shard's tiles in the
   * grouped order of its mq tile rows. */
  int32_t const mq = m_tiles / n_pes;
  int32_t const per_shard = mq * n_tiles;
  int32_t const d = r / per_shard;
  int32_t row, col;
  out[3] = r - d * per_shard;
  out[2] = (my_pe + d) % n_pes;
  grouped_raster(out[3], mq, n_tiles, group_m < mq ? group_m : mq, &row, &col);
  out[0] = out[2] * mq + row;
  out[1] = col;
}

int32_t oracle_gather_chunk_rows(int64_t k) {
  int32_t rows = 128;
  while (rows > 1 && (int64_t)rows * k * 2 > 65536) rows /= 2;
  return rows;
}

int64_t oracle_gather_events_words(int32_t n_pes, int32_t tiles, int32_t mq) {
  /* arrive[2][1][tiles][4], ready[n_pes], read_done[n_pes], rows[n_pes][mq],
   * chunks[n_pes] */
  return (int64_t)2 * tiles * 4 + 3 * (int64_t)n_pes + (int64_t)n_pes * mq;
}

int oracle_allgather_gemm(const oracle_bf16_problem *p, const float *const *a_shard,
                          const float *const *b, float *const *gathered, float *const *out,
                          uint32_t *const *events, uint64_t *counters,
                          int32_t *const *gemm_order) {
  int32_t const np = p->n_pes;
  int64_t const m = p->m, n = p->n, k = p->k;
  int64_t const rows_per_pe = m / np;
  int32_t const mt = (int32_t)(m / p->tile_m);
  int32_t const nt = (int32_t)((n + p->tile_n - 1) / p->tile_n);
  int32_t const tiles = mt * nt;
  int32_t const mq = mt / np;
  uint32_t const epoch = p->epoch;
  int32_t const parity = (int32_t)(epoch & 1u);
  int32_t const chunks_per_block = p->tile_m / oracle_gather_chunk_rows(k);
  int64_t const gw = (int64_t)2 * tiles * 4; /* first word of the gather region */
  uint64_t local_counters[8 * 8];
  uint64_t *cnt = counters != NULL ? counters : local_counters;
  if (m % ((int64_t)np * p->tile_m) != 0) return -1;
  memset(cnt, 0, sizeof(uint64_t) * 8 * (size_t)np);

  for (int32_t pe = 0; pe < np; ++pe) {
    /* Every PE announces its shard; every other PE copies all of it
     * (chunks of whole rows), counting chunks per tile row, then tells the
     * shard's owner; the counters are zeroed at the end of the launch. */
    for (int32_t src = 0; src < np; ++src) {
      memcpy(gathered[pe] + src * rows_per_pe * k, a_shard[src],
             sizeof(float) * (size_t)(rows_per_pe * k));
      if (events && src != pe) {
        events[pe][gw + src] = epoch;      /* ready[src], set by src */
        events[src][gw + np + pe] = epoch; /* read_done[pe] on src, set by pe */
      }
    }
    cnt[pe * 8 + 1] += (uint64_t)np * mq * chunks_per_block;
    cnt[pe * 8 + 4] += (uint64_t)(np - 1);
    cnt[pe * 8 + 5] += (uint64_t)(np - 1);
    if (events) {
      for (int64_t w = 0; w < (int64_t)np * mq + np; ++w) events[pe][gw + 2 * np + w] = 0;
    }
    oracle_gemm_f32(gathered[pe], b[pe], out[pe], m, n, k, p->threads);
    /* GEMM tiles in PE pe's raster order, each quarter published locally. */
    for (int32_t r = 0; r < tiles; ++r) {
      int32_t c[4];
      oracle_locate_gather(mt, nt, np, pe, p->group_m, r, c);
      int32_t const t = c[0] * nt + c[1];
      if (gemm_order) gemm_order[pe][r] = t;
      cnt[pe * 8 + 0] += 1;
      if (c[2] != pe) cnt[pe * 8 + 3] += 1;
      for (int32_t q = 0; q < 4; ++q) {
        if (events) events[pe][arrive_idx(parity, 0, t, q, 1, tiles)] = epoch;
        cnt[pe * 8 + 2] += 1;
      }
    }
    cnt[pe * 8 + 6] += 1;
  }
  return 0;
}

/* ---- single-launch MLP chain: event words and counters (a B200 addition;
 *      restates chain_kernel.cuh's layout and publish rules) ------------- */

static int32_t chain_quarters(int32_t row, int64_t tokens) {
  int64_t const left = tokens - (int64_t)row * 128;
  int64_t const q = (left + 31) / 32;
  return (int32_t)(q < 4 ? q : 4);
}

int64_t oracle_chain_events_words(int32_t layers, int32_t n_pes, int64_t tokens,
                                  int64_t hidden) {
  int64_t const mt = (tokens + 127) / 128, dn = (hidden + 255) / 256;
  return (int64_t)layers * n_pes * mt * dn * 4 + 2 * (int64_t)layers * mt;
}

void oracle_chain_events(int32_t layers, int32_t n_pes, int64_t tokens, int64_t hidden,
                         int64_t inter, int32_t group_m, uint32_t epoch,
                         uint32_t *const *events, uint64_t *counters) {
  int32_t const mt = (int32_t)((tokens + 127) / 128);
  int32_t const gn = (int32_t)((inter + 127) / 128);  /* act columns per GU tile: 128 */
  int32_t const dn = (int32_t)((hidden + 255) / 256); /* hidden columns per DN tile: 256 */
  int32_t const tiles = mt * dn;
  int64_t const counters_base = (int64_t)layers * n_pes * tiles * 4;
  int64_t quarters = 0;
  for (int32_t row = 0; row < mt; ++row) quarters += chain_quarters(row, tokens);
  memset(counters, 0, sizeof(uint64_t) * 8 * (size_t)n_pes);
  for (int32_t pe = 0; pe < n_pes; ++pe) {
    uint64_t *c = counters + 8 * pe;
    c[0] = (uint64_t)layers * mt * (gn + dn);                 /* GEMM tiles */
    c[2] = (uint64_t)layers * (uint64_t)quarters * (gn + dn); /* quarter publishes */
    c[6] = 1;
    for (int32_t l = 0; l < layers; ++l) {
      for (int32_t row = 0; row < mt; ++row) {
        int32_t const aq = chain_quarters(row, tokens);
        /* act_ready: every GU quarter of the row; x_ready: every (DN tile,
         * quarter) of the row, counted by its owner (or the epilogue on one
         * PE). The host zeroes both before the launch. */
        events[pe][counters_base + (int64_t)l * mt + row] = (uint32_t)(aq * gn);
        events[pe][counters_base + (int64_t)(layers + l) * mt + row] = (uint32_t)(aq * dn);
      }
    }
    if (n_pes == 1) continue;
    c[5] = (uint64_t)n_pes; /* the final wait, once per call */
    for (int32_t r = 0; r < tiles; ++r) {
      int32_t loc[4];
      oracle_locate(mt, dn, n_pes, 0, group_m, r, loc);
      if (loc[2] != pe) continue;
      int32_t const t = loc[0] * dn + loc[1];
      int32_t const aq = chain_quarters(loc[0], tokens);
      c[1] += (uint64_t)layers * aq;          /* exchange sub-tasks */
      c[3] += (uint64_t)layers * aq * n_pes;  /* partial acquires */
      c[4] += (uint64_t)layers * aq * n_pes;  /* final stores counted per PE */
      /* every PE's partial of every active quarter of an owned tile */
      for (int32_t l = 0; l < layers; ++l)
        for (int32_t src = 0; src < n_pes; ++src)
          for (int32_t q = 0; q < aq; ++q)
            events[pe][(((int64_t)l * n_pes + src) * tiles + t) * 4 + q] = epoch;
    }
  }
}

/* ---- CPU-baseline sample: a list of output tiles -------------------------- */

typedef struct tile_job {
  const oracle_bf16_problem *p;
  const float *const *a;
  const float *const *b;
  const int32_t *tile_ids;
  int32_t first, last;
  float *out;
} tile_job;

static void *tile_worker(void *arg) {
  tile_job *j = (tile_job *)arg;
  const oracle_bf16_problem *p = j->p;
  int64_t const n = p->n, m = p->m;
  int32_t const nt = (int32_t)((n + p->tile_n - 1) / p->tile_n);
  float *scratch = (float *)malloc(sizeof(float) * (size_t)(p->tile_m * n));
  for (int32_t i = j->first; i < j->last; ++i) {
    int32_t const t = j->tile_ids[i];
    int64_t const r0 = (int64_t)(t / nt) * p->tile_m, c0 = (int64_t)(t % nt) * p->tile_n;
    int64_t const r1 = r0 + p->tile_m < m ? r0 + p->tile_m : m;
    int64_t const c1 = c0 + p->tile_n < n ? c0 + p->tile_n : n;
    for (int64_t r = r0; r < r1; ++r)
      for (int64_t c = c0; c < c1; ++c) j->out[r * n + c] = 0.0f;
    for (int32_t pe = 0; pe < p->n_pes; ++pe) {
      /* Partial rows [r0, r1) of PE pe, computed into a row-offset scratch. */
      oracle_gemm_block(j->a[pe] + r0 * p->k, j->b[pe], scratch, r1 - r0, n, p->k, 0, r1 - r0, c0,
                        c1);
      for (int64_t r = r0; r < r1; ++r) {
        for (int64_t c = c0; c < c1; ++c) {
          float v = scratch[(r - r0) * n + c];
          if (p->n_pes > 1 && p->wire_bytes == 2) v = oracle_round_bf16(v);
          j->out[r * n + c] += v;
        }
      }
    }
  }
  free(scratch);
  return NULL;
}

void oracle_bf16_tiles(const oracle_bf16_problem *p, const float *const *a,
                       const float *const *b, const int32_t *tile_ids, int32_t n_listed,
                       float *out_full) {
  int32_t threads = p->threads > 0 ? p->threads : 1;
  if (threads > n_listed) threads = n_listed > 0 ? n_listed : 1;
  pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
  tile_job *jobs = (tile_job *)malloc(sizeof(tile_job) * (size_t)threads);
  for (int32_t t = 0; t < threads; ++t) {
    jobs[t].p = p;
    jobs[t].a = a;
    jobs[t].b = b;
    jobs[t].tile_ids = tile_ids;
    jobs[t].first = n_listed * t / threads;
    jobs[t].last = n_listed * (t + 1) / threads;
    jobs[t].out = out_full;
    pthread_create(&tid[t], NULL, tile_worker, &jobs[t]);
  }
  for (int32_t t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(jobs);
  free(tid);
}

/* ---- tensor-parallel MLP blocks -------------------------------------------- */

void oracle_mlp_chain(int64_t t, int64_t h, int64_t i, int32_t layers, int32_t n_pes,
                      int32_t wire_bytes, const float *x, const float *const *wg,
                      const float *const *wu, const float *const *wd, float *out,
                      int32_t threads) {
  float *cur = (float *)malloc(sizeof(float) * (size_t)(t * h));
  float *g = (float *)malloc(sizeof(float) * (size_t)(t * i));
  float *u = (float *)malloc(sizeof(float) * (size_t)(t * i));
  float *part = (float *)malloc(sizeof(float) * (size_t)(t * h));
  float *sum = (float *)malloc(sizeof(float) * (size_t)(t * h));
  memcpy(cur, x, sizeof(float) * (size_t)(t * h));
  for (int32_t l = 0; l < layers; ++l) {
    for (int64_t e = 0; e < t * h; ++e) sum[e] = 0.0f;
    for (int32_t p = 0; p < n_pes; ++p) {
      int64_t const w = (int64_t)l * n_pes + p;
      oracle_gemm_f32(cur, wg[w], g, t, i, h, threads);
      oracle_gemm_f32(cur, wu[w], u, t, i, h, threads);
      for (int64_t e = 0; e < t * i; ++e) {
        float const s = g[e] / (1.0f + expf(-g[e]));
        g[e] = oracle_round_bf16(s * u[e]); /* act */
      }
      oracle_gemm_f32(g, wd[w], part, t, h, i, threads);
      for (int64_t e = 0; e < t * h; ++e) {
        sum[e] += wire_bytes == 2 ? oracle_round_bf16(part[e]) : part[e];
      }
    }
    for (int64_t e = 0; e < t * h; ++e) cur[e] = oracle_round_bf16(sum[e]);
  }
  memcpy(out, cur, sizeof(float) * (size_t)(t * h));
  free(cur);
  free(g);
  free(u);
  free(part);
  free(sum);
}
