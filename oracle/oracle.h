/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle of the fused GEMM + allreduce /
 * reduce-scatter path. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline legs may load it, and only as the checker or the timed CPU
 * baseline; the product path never calls it.
 *
 * It restates, in plain C, megacu's tile-task graph:
 *   - the fp32 tile GEMM with k ascending, one fused multiply-add per step
 *     (golden/golden_gemm_allreduce.cu:65-98,
 *      phased/megacu/megacu_gemm_allreduce_phased.cu:56-89);
 *   - the reduction out = sum over PEs in PE order 0..n-1, fp32
 *     (golden_gemm_allreduce.cu:192-240, megacu_gemm_allreduce_phased.cu:91-133);
 *   - the event tensor int32 [n_pes][tiles], slot = pe * tiles + tile, ready
 *     value tile + 1 (backends/nvshmem/cuda_event_tensor.cuh:13-58);
 * and, for the B200 megakernel, the same graph with the device task queue's
 * raster order, the tile ownership of two-shot / one-shot allreduce and
 * reduce-scatter, and the epoch-tagged quarter-tile event tensor (restated
 * from megacu_b200/csrc/kernels/tile_schedule.h and layout.h).
 *
 * Parity pins: the reference's known-answer tests
 * (tests/runtime/cuda_gemm_allreduce_correctness.cc:92-99 and
 *  tests/runtime/nvshmem_two_rank_smoke.cc:101-102) are committed as
 * fixtures in tests/golden/ and checked by tests/test_oracle.py.
 */
#ifndef MEGACU_B200_ORACLE_H_
#define MEGACU_B200_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* c[m, n] = a[m, k] @ b[k, n], fp32, k ascending with fmaf per step, rows
 * split over `threads` POSIX threads (the order per element is unchanged). */
void oracle_gemm_f32(const float *a, const float *b, float *c, int64_t m, int64_t n,
                     int64_t k, int32_t threads);

/* The same for the sub-block rows [r0, r1) x cols [c0, c1) of c (ldc = n). */
void oracle_gemm_block(const float *a, const float *b, float *c, int64_t m, int64_t n,
                       int64_t k, int64_t r0, int64_t r1, int64_t c0, int64_t c1);

/* Round-to-nearest-even fp32 -> bf16 -> fp32. */
float oracle_round_bf16(float x);

/*
 * megacu's phased fp32 graph on n_pes logical PEs (one call):
 * per PE: GEMM tiles in tile-id order publish events[pe][tile] = tile + 1 on
 * every PE; every PE then acquires all PEs' slot of each tile and sums the
 * partials in PE order into its out. a[pe]: [m, k], b[pe]: [k, n],
 * out[pe]: [m, n]; events[pe]: int32 [n_pes][tiles] (reset by the call).
 * Returns 0, or a negative number if an acquire found a slot unset.
 */
int oracle_phased_f32(int64_t m, int64_t n, int64_t k, int32_t tile_m, int32_t tile_n,
                      int32_t n_pes, const float *const *a, const float *const *b,
                      float *const *out, int32_t *const *events);

/* Tile schedule restatement: raster index r -> out[0] tile row, out[1] tile
 * column, out[2] owner PE, out[3] index among the owner's tiles. */
void oracle_locate(int32_t m_tiles, int32_t n_tiles, int32_t n_pes, int32_t mode,
                   int32_t group_m, int32_t r, int32_t out[4]);

/*
 * Tensor-parallel MLP blocks (benchmark config 5; a B200 addition with no
 * counterpart in megacu, so its semantics are pinned by this restatement):
 * for l = 0 .. layers-1, on every PE p,
 *   act_p = bf16(silu(x_l @ wg[l][p]) * (x_l @ wu[l][p]))   (fp32 products and
 *            epilogue, silu(g) = g / (1 + expf(-g)), one bf16 rounding)
 *   x_{l+1} = bf16(sum over p = 0..n_pes-1 of wire(act_p @ wd[l][p]))
 * with wire() rounding each partial to bf16 when wire_bytes == 2 (fp32 sum
 * in PE order either way). x: [t, h]; wg, wu: [h, i] per layer and PE (index
 * l * n_pes + p); wd: [i, h]; out: [t, h] = x_layers. Inputs are bf16 values
 * held as fp32.
 */
void oracle_mlp_chain(int64_t t, int64_t h, int64_t i, int32_t layers, int32_t n_pes,
                      int32_t wire_bytes, const float *x, const float *const *wg,
                      const float *const *wu, const float *const *wd, float *out,
                      int32_t threads);

/*
 * Event words and completion counters of one single-launch MLP chain call
 * (a B200 addition; restates chain_kernel.cuh): events[pe] holds the words
 * after the control block, oracle_chain_events_words() of them; arrive flags
 * [layer][src][DN tile][quarter] of the tiles PE pe owns are set to `epoch`
 * (other words are left as they are), the act_ready / x_ready counters hold
 * their values after the call. counters[pe * 8 + i] receive the per-call
 * deltas of the device counters. group_m is the DN raster's band height.
 */
int64_t oracle_chain_events_words(int32_t layers, int32_t n_pes, int64_t tokens, int64_t hidden);
void oracle_chain_events(int32_t layers, int32_t n_pes, int64_t tokens, int64_t hidden,
                         int64_t inter, int32_t group_m, uint32_t epoch,
                         uint32_t *const *events, uint64_t *counters);

/* CTA-pair schedule restatement (a B200 addition with no counterpart in
 * megacu): GEMM pair ticket q -> out[0], out[1] = raster indices of the
 * upper and lower 128-row tiles the two CTAs of a cluster compute. */
void oracle_pair_raster(int32_t n_pes, int32_t mode, int32_t q, int32_t out[2]);

typedef struct oracle_bf16_problem {
  int64_t m, n, k;       /* k = per-PE slice */
  int32_t tile_m;        /* 128 */
  int32_t tile_n;        /* 64 / 128 / 256 */
  int32_t n_pes;
  int32_t mode;          /* 0 allreduce, 1 reduce-scatter */
  int32_t one_shot;
  int32_t group_m;       /* raster band height */
  int32_t wire_bytes;    /* 2: partials rounded to bf16 before the sum; 4: fp32 */
  int32_t threads;       /* CPU threads for the GEMMs */
  uint32_t epoch;        /* the call's epoch tag (launch count + 1) */
} oracle_bf16_problem;

/*
 * The B200 megakernel's tile-task graph for one call on n_pes logical PEs.
 * a[pe], b[pe]: bf16 values held in fp32. out[pe]: fp32 result, [m, n] for
 * allreduce, [m / n_pes, n] for reduce-scatter (not rounded to bf16).
 * events[pe] (optional): the event tensor words after the control block —
 * arrive uint32 [2][n_pes][tiles][4] then done uint32 [2][n_pes] — updated in
 * place exactly as the device does. counters[pe * 8 + i]
 * (optional) receive the per-call deltas of the device counters. gemm_order
 * (optional, [tiles]) receives the tile id of each GEMM ticket;
 * reduce_order[pe] (optional, [tiles * 4 * tile_n / 64]) the tile id of each
 * reduce ticket (reduced tile in raster order, 32-row quarter, 64-column
 * block) of PE pe, or -1 where the block holds no output element.
 * Returns 0, or a negative number if the graph was inconsistent (an acquire
 * found a flag unset).
 */
int oracle_bf16_call(const oracle_bf16_problem *p, const float *const *a,
                     const float *const *b, float *const *out, uint32_t *const *events,
                     uint64_t *counters, int32_t *gemm_order, int32_t *const *reduce_order);

/*
 * All-gather + GEMM (a B200 addition with no counterpart in megacu, pinned by
 * this restatement): on every PE p of n_pes, gathered[p] = the a_shard of
 * every PE stacked in PE order ([m, k], m = n_pes * rows per shard) and
 * out[p] = gathered[p] @ b[p] ([m, n], fp32 with k ascending, not rounded).
 * p->m must be a multiple of n_pes * tile_m; mode, one_shot and wire_bytes
 * are ignored. events[p] (optional): the words after the control block —
 * arrive[2][1][tiles][4], ready[n_pes], read_done[n_pes], rows[n_pes][mq],
 * chunks[n_pes] — as the device leaves them after the call (the two counter
 * arrays zeroed). counters[p * 8 + i] receive the per-call deltas;
 * gemm_order[p] (optional, [tiles]) the tile id of each of PE p's GEMM
 * tickets. Returns 0, or -1 if m is not a multiple of n_pes * tile_m.
 */
int oracle_allgather_gemm(const oracle_bf16_problem *p, const float *const *a_shard,
                          const float *const *b, float *const *gathered, float *const *out,
                          uint32_t *const *events, uint64_t *counters,
                          int32_t *const *gemm_order);

/* All-gather raster of PE my_pe: r -> out[0] tile row, out[1] tile column,
 * out[2] the PE whose shard holds the rows, out[3] index within that shard. */
void oracle_locate_gather(int32_t m_tiles, int32_t n_tiles, int32_t n_pes, int32_t my_pe,
                          int32_t group_m, int32_t r, int32_t out[4]);

/* Rows per all-gather copy chunk for a given K (about 64 KiB, a power of two
 * dividing 128), and the gather event words after the control block. */
int32_t oracle_gather_chunk_rows(int64_t k);
int64_t oracle_gather_events_words(int32_t n_pes, int32_t tiles, int32_t mq);

/*
 * CPU-baseline sample: the summed output of the listed tiles only (full K
 * on every PE, PE-order fp32 sum), written into out_full[m, n] at the tiles'
 * positions. Uses `threads` POSIX threads across the listed tiles.
 */
void oracle_bf16_tiles(const oracle_bf16_problem *p, const float *const *a,
                       const float *const *b, const int32_t *tile_ids, int32_t n_tiles_listed,
                       float *out_full);

#ifdef __cplusplus
}
#endif

#endif /* MEGACU_B200_ORACLE_H_ */
