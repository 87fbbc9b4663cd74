/*
 * megacu_b200 C ABI: the binary drop-in boundary of the fused
 * GEMM + allreduce / reduce-scatter megakernel for B200 (sm_100a).
 *
 * Plain C: only pointers, sizes and POD structs cross this boundary. The
 * structs below are layout-identical to megacu's C++ types so that a caller
 * compiled against megacu's headers can bind these symbols directly:
 *   megacu_status        == megacu::status          (views.h:27-31)
 *   megacu_driver_view   == megacu::cuda_nvshmem::driver_view (runtime.h:416-419)
 *   megacu_gemm_ar_problem == gemm_ar_problem       (examples/cuda_nvshmem/
 *                                                    gemm_allreduce/common/
 *                                                    gemm_allreduce.h:26-32)
 *
 * Conventions (same as megacu's launcher, megacu_gemm_allreduce_phased.cu:157-232):
 *  - every call returns a status by value and never throws;
 *  - the caller owns every buffer; nothing here allocates per call;
 *  - a launch is asynchronous on driver.launch.stream; a null stream means
 *    "validate only" and returns ok without touching the GPU;
 *  - with team_n_pes > 1 every PE calls collectively, in the same order.
 */
#ifndef MEGACU_B200_H_
#define MEGACU_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status and views (layout of megacu::status / driver_view) ---------- */

enum megacu_status_code {
  MEGACU_OK = 0,
  MEGACU_INVALID_ARGUMENT = 1,
  MEGACU_UNSUPPORTED = 2,
  MEGACU_BACKEND_ERROR = 3,
  MEGACU_LAUNCH_ERROR = 4
};

typedef struct megacu_status {
  uint8_t code;        /* enum megacu_status_code */
  uint16_t detail;     /* per-call-site number */
  const char *message; /* static string, never freed */
} megacu_status;

/*
 * Detail numbers. megacu's own: 1 invalid problem or argument value,
 * 2 missing storage or output pointer, 10 cudaSetDevice / device ordinal,
 * 11 memset, 12 team barrier launch, 13 remote PEs without a megacu_b200 team,
 * 14 kernel launch. B200 additions:
 *   20 dtype is not bf16            21 n, k or a buffer not 16-byte aligned
 *   22 unsupported size or tile     23 team size / PE index out of range
 *   24 team handle does not match   25 buffer outside the symmetric heap
 *   26 reduce-scatter or all-gather m not a multiple of tp * 128
 *   27 CTA pairs requested but the tile grid cannot hold them
 *   28 in-switch reduction not possible: the fp32 wire with the workspace in
 *      the multicast region, or a two-shot allreduce with only one of
 *      workspace and out there
 *   29 outside a single-launch MLP chain's limits (more than 6 blocks, or
 *      the fp32 wire)
 *   30 cuTensorMapEncodeTiled failed
 *   31 exporting the team heap (CUDA IPC), 32 peer handle of another team,
 *   33 peer mapping (CUDA IPC / peer access), 34 symmetric heap exhausted
 *   35 no multicast region possible (device, driver, one PE, shared process)
 *   36 multicast region set-up out of order, 37 multicast driver call,
 *   38 multicast object export / hand-over
 *   39 local rendezvous failed or timed out (megacu_b200_exchange_local)
 *   40 a cross-GPU wait timed out, 41 a local pipeline wait timed out,
 *   42 a kernel bounds check failed (only in the bounds-checked build,
 *      libmegacu_b200_checked.so) (megacu_b200_events_status)
 *   50 built-in scratch address lookup, 51 more than one PE,
 *   52 tile grid larger than the built-in scratch (megacu_cuda_gemm_bf16_noalloc)
 */

typedef struct megacu_launch_view {
  void *stream; /* cudaStream_t; NULL = validate only */
  int32_t device_ordinal;
} megacu_launch_view;

typedef struct megacu_team_view {
  void *team; /* megacu_b200_team handle when team_n_pes > 1, else NULL */
  int32_t team_my_pe;
  int32_t team_n_pes;
  int32_t world_my_pe;
  int32_t world_n_pes;
  int32_t cuda_device_ordinal;
  uint16_t backend;
  uint64_t session;
  uint8_t owner;
} megacu_team_view;

typedef struct megacu_driver_view {
  megacu_launch_view launch;
  megacu_team_view team;
} megacu_driver_view;

/* megacu's problem descriptor (fp32 launcher). */
typedef struct megacu_gemm_ar_problem {
  int64_t m;
  int64_t n;
  int64_t k;
  int32_t tile_m;
  int32_t tile_n;
} megacu_gemm_ar_problem;

/* ---- bf16 problem descriptor (new; no counterpart in megacu) ------------- */

enum megacu_gemm_ar_mode {
  MEGACU_MODE_ALLREDUCE = 0,      /* out[m, n] on every PE */
  MEGACU_MODE_REDUCE_SCATTER = 1, /* PE p holds rows [p*m/tp, (p+1)*m/tp) */
  MEGACU_MODE_ALLGATHER = 2       /* A gathered along M before the GEMM
                                     (megacu_cuda_allgather_gemm_bf16) */
};

enum megacu_gemm_ar_algo {
  MEGACU_ALGO_AUTO = 0,
  MEGACU_ALGO_ONE_SHOT = 1, /* every PE reads every PE's partial of every
                               tile and reduces it into its own out */
  MEGACU_ALGO_TWO_SHOT = 2  /* the tile's owner reads every PE's partial,
                               reduces, and stores the sum into every PE's out */
};

/* How GEMM tiles map to CTAs. With pairs, the two CTAs of a 2-CTA cluster
 * (two SMs) compute two vertically adjacent 128-row tiles together with
 * 256-row tcgen05 MMAs, each SM staging half of the B tile; events,
 * ownership and partial slots stay per 128-row tile. Pairs need an even
 * number of tile rows (per PE block in reduce-scatter) and tile_n >= 128. */
enum megacu_cta_pairs {
  MEGACU_CTA_PAIRS_AUTO = 0,  /* pairs whenever the tile grid allows them */
  MEGACU_CTA_PAIRS_OFF = 1,   /* one CTA per tile */
  MEGACU_CTA_PAIRS_ON = 2     /* pairs, or MEGACU_UNSUPPORTED if not possible */
};

/* Element type codes, numbered as megacu::dtype (views.h:12-17). */
enum megacu_dtype {
  MEGACU_DTYPE_UNKNOWN = 0,
  MEGACU_DTYPE_F16 = 1,
  MEGACU_DTYPE_BF16 = 2,
  MEGACU_DTYPE_F32 = 3
};

typedef struct megacu_gemm_ar_problem_v2 {
  int64_t m;             /* rows of A and of the full output */
  int64_t n;             /* columns of B and of the output; multiple of 8 */
  int64_t k;             /* this PE's slice of K; multiple of 8 */
  int32_t tile_m;        /* 0 = auto (128) */
  int32_t tile_n;        /* 0 = auto; else 64, 128 or 256 */
  int32_t mode;          /* enum megacu_gemm_ar_mode */
  int32_t algo;          /* enum megacu_gemm_ar_algo */
  int32_t deterministic; /* 1 = partials cross NVLink as fp32 (one bf16
                            rounding in total); 0 = as bf16. The rank-order
                            fp32 reduction is fixed in both modes, so both are
                            bit-reproducible run to run. */
  int32_t dtype;         /* must be MEGACU_DTYPE_BF16 */
  int32_t num_ctas;      /* 0 = one persistent CTA per SM */
  int32_t cta_pairs;     /* enum megacu_cta_pairs */
  uint64_t timeout_ns;   /* bound of every cross-GPU wait; 0 = 10 s */
  uint64_t *trace;       /* optional device buffer of trace records, NULL =
                            off: 4 x uint64 {kind | sub << 8 | CTA << 16 |
                            ticket << 32, tile, start ns, end ns}; kinds 0
                            GEMM tile epilogue, 2 reduce sub-task, 3 worker
                            completion fence, 4 done flags stored, 5 wait
                            for every PE's done flag, 6 all-gather copy
                            chunk (sub = hops to its shard's PE, tile =
                            shard * (m / tp / 128) + tile row) */
  int64_t trace_capacity; /* records that fit in `trace` */
} megacu_gemm_ar_problem_v2;

/* ---- megacu's fp32 phased launcher (binary drop-in) ---------------------- */

/*
 * Replaces megacu `megacu_cuda_gemm_allreduce_phased_f32`
 * (examples/cuda_nvshmem/gemm_allreduce/phased/megacu/
 *  megacu_gemm_allreduce_phased.cu:157-232; declared at
 *  common/gemm_allreduce_orchestrate_common.h:8-11).
 * out[m, n] = sum over PEs of a_pe[m, k] * b_pe[k, n], fp32, row-major.
 * `partial` (>= m*n floats) and `events` (>= tiles*n_pes int32) must lie in
 * the team's symmetric heap when team_n_pes > 1. Events are reset by the call.
 */
megacu_status megacu_cuda_gemm_allreduce_phased_f32(
    megacu_driver_view driver, const float *a, const float *b, float *partial,
    float *out, void *events, megacu_gemm_ar_problem problem);

/* ---- bf16 fused megakernel (north-star path) ----------------------------- */

/*
 * Tensor-parallel bf16 GEMM (fp32 accumulate) fused with the allreduce of
 * the per-PE partial products: out[m, n] = sum_pe a_pe[m, k] @ b_pe[k, n].
 * a: row-major [m, k] bf16; b: row-major [k, n] bf16; out: row-major [m, n]
 * bf16, in the symmetric heap when team_n_pes > 1.
 * workspace: >= megacu_b200_workspace_bytes(); symmetric when team_n_pes > 1.
 * events: >= megacu_b200_events_bytes(); symmetric when team_n_pes > 1,
 * zero-filled once before first use, then reused across calls without reset.
 * Replaces the same role as megacu_gemm_allreduce_phased.cu:157-232, for bf16.
 */
megacu_status megacu_cuda_gemm_allreduce_bf16(
    megacu_driver_view driver, const void *a, const void *b, void *workspace,
    void *out, void *events, megacu_gemm_ar_problem_v2 problem);

/*
 * Same GEMM fused with a reduce-scatter along M: PE p receives rows
 * [p*m/tp, (p+1)*m/tp) of the sum in `out` (row-major [m/tp, n] bf16, local
 * memory). m must be a multiple of tp * tile_m.
 */
megacu_status megacu_cuda_gemm_reduce_scatter_bf16(
    megacu_driver_view driver, const void *a, const void *b, void *workspace,
    void *out, void *events, megacu_gemm_ar_problem_v2 problem);

/*
 * All-gather of A along M fused with the GEMM that consumes it (the
 * sequence-parallel input of a column-parallel projection; new, no
 * counterpart in megacu):
 *   gathered[m, k] = every PE's a_shard stacked in PE order
 *   out[m, n]      = gathered @ b (fp32 accumulate, one bf16 rounding)
 * problem: m = total rows (a multiple of tp * 128), n = this PE's columns
 * (multiple of 8), k = the full K (multiple of 8); mode is set to
 * MEGACU_MODE_ALLGATHER; `deterministic` has no effect (nothing is summed
 * across PEs). a_shard: row-major [m/tp, k] bf16 in the team's symmetric
 * heap when team_n_pes > 1 (the peers copy it over NVLink); b: [k, n];
 * gathered: [m, k]; out: [m, n]; all three local. events:
 * megacu_b200_events_bytes() with mode MEGACU_MODE_ALLGATHER, symmetric,
 * zero-filled once. No workspace. Inside the launch, worker warps copy the
 * peers' shards (peer loads, the nearest PEs first) into `gathered` while
 * the GEMM computes the tiles of rows already present, each tile row
 * released by a counter of its copied chunks; the call ends once every
 * peer has copied this PE's shard, so a_shard may be rewritten by the next
 * stream-ordered work. Event tensor: arrive[p][0][t][q] = epoch per stored
 * tile quarter; counters[1] counts copy chunks, [3] tiles that waited for
 * gathered rows, [4] / [5] the "shard copied" flags sent / acquired.
 */
megacu_status megacu_cuda_allgather_gemm_bf16(
    megacu_driver_view driver, const void *a_shard, const void *b, void *gathered,
    void *out, void *events, megacu_gemm_ar_problem_v2 problem);

/* ---- tensor-parallel MLP blocks (benchmark config 5; new, no counterpart in
 *      megacu) -------------------------------------------------------------- */

/*
 * Column-parallel gate/up projection with the SwiGLU epilogue, one PE:
 * act[m, n] = bf16(silu(x @ w_gate) * (x @ w_up)), the products accumulated in
 * fp32 and the epilogue computed in fp32 (silu(g) = g / (1 + exp(-g))).
 * x: row-major [m, k]; w_gate, w_up: row-major [k, n] (this PE's column
 * slice); act: row-major [m, n], local. problem.m = tokens, n = this PE's
 * intermediate columns, k = hidden; tile_n must be 0 (auto: 128 act columns,
 * i.e. 128 gate + 128 up accumulator columns per tile). events: >=
 * megacu_b200_swiglu_events_bytes(), local, zero-filled once.
 */
megacu_status megacu_cuda_gemm_swiglu_bf16(
    megacu_driver_view driver, const void *x, const void *w_gate, const void *w_up,
    void *act, void *events, megacu_gemm_ar_problem_v2 problem);
megacu_status megacu_b200_swiglu_events_bytes(megacu_gemm_ar_problem_v2 problem,
                                              int64_t *bytes);

typedef struct megacu_mlp_chain_problem {
  int64_t tokens;        /* rows of x and of every block's output */
  int64_t hidden;        /* columns of x; multiple of 8 */
  int64_t inter;         /* this PE's slice of the intermediate size; multiple of 8 */
  int32_t layers;        /* MLP blocks, 1..64 */
  int32_t algo;          /* allreduce algo of the down projection */
  int32_t deterministic; /* as in megacu_gemm_ar_problem_v2 */
  int32_t num_ctas;      /* 0 = one persistent CTA per SM */
  int32_t cta_pairs;     /* enum megacu_cta_pairs, every launch */
  int32_t single_launch; /* 0: two launches per block; 1: all blocks (at most
                            6) in one persistent launch, blocks waiting for
                            each other through counters in events_down
                            (bf16 partials, two-shot peer exchange) */
  uint64_t timeout_ns;   /* bound of every cross-GPU wait; 0 = 10 s */
} megacu_mlp_chain_problem;

/*
 * Buffer sizes of megacu_cuda_mlp_chain_bf16 on `n_pes` PEs: sizes[0] act
 * (local), [1] workspace (symmetric), [2] events_swiglu (local), [3]
 * events_down (symmetric), [4] x_work (like out).
 */
megacu_status megacu_b200_mlp_chain_sizes(megacu_mlp_chain_problem problem, int32_t n_pes,
                                          int64_t sizes[5]);

/*
 * `layers` tensor-parallel MLP blocks back to back, every PE collectively:
 *   act = silu(x_l @ w_gate[l]) * (x_l @ w_up[l])           (local)
 *   x_{l+1} = sum over PEs of act @ w_down[l]               (fused allreduce)
 * x_0 = x: row-major [tokens, hidden], local. w_gate[l], w_up[l]: [hidden,
 * inter]; w_down[l]: [inter, hidden] (host arrays of `layers` device
 * pointers to this PE's slices). The blocks' outputs alternate between out
 * and x_work so that the last one lands in out; both are placed like the
 * out of megacu_cuda_gemm_allreduce_bf16 (symmetric for two-shot; in the
 * team's multicast region, together with workspace, for the in-switch
 * reduction). With single_launch = 0, two launches per block:
 * megacu_cuda_gemm_swiglu_bf16, then megacu_cuda_gemm_allreduce_bf16. With
 * single_launch = 1, one persistent launch runs every block; workspace, out,
 * x_work and events_down then lie in the team's heap (not its multicast
 * region). One events_down buffer serves either mode.
 */
megacu_status megacu_cuda_mlp_chain_bf16(
    megacu_driver_view driver, const void *x, const void *const *w_gate,
    const void *const *w_up, const void *const *w_down, void *act, void *workspace,
    void *x_work, void *out, void *events_swiglu, void *events_down,
    megacu_mlp_chain_problem problem);

/*
 * Orchestrated entry: builds megacu's three-task phase (GEMM tile producer
 * with tile_grid + publish, sync with join, reduce consumer with acquire),
 * validates it with the dispatcher and ASAP scheduler, then calls the bf16
 * launcher above (mode taken from problem.mode). Mirrors megacu
 * `cuda_nvshmem_gemm_allreduce_phased_orchestrate`
 * (phased/megacu/gemm_allreduce_phased_orchestrate.cc:3-20).
 */
megacu_status megacu_cuda_gemm_allreduce_bf16_orchestrate(
    megacu_driver_view driver, const void *a, const void *b, void *workspace,
    void *out, void *events, megacu_gemm_ar_problem_v2 problem);

/*
 * C-linkage form of megacu's fp32 orchestrate entry
 * `cuda_nvshmem_gemm_allreduce_phased_orchestrate`
 * (phased/megacu/gemm_allreduce_phased_orchestrate.cc:3-20): builds the same
 * three-task phase, validates it, runs megacu_cuda_gemm_allreduce_phased_f32.
 * The C++-linkage original is declared in <megacu/gemm_allreduce.h>.
 */
megacu_status megacu_cuda_gemm_allreduce_f32_orchestrate(
    megacu_driver_view driver, const float *a, const float *b, float *partial,
    float *out, void *events, megacu_gemm_ar_problem problem);

/*
 * megacu's fp32 phase with co-resident persistent progress (a B200
 * extension). megacu declares progress_model::co_resident_persistent
 * (include/megacu/runtime.h:18) but its scheduler rejects it
 * (src/scheduler/explicit_asap.cc:34-39). This entry builds the same
 * three-task phase as cuda_nvshmem_gemm_allreduce_phased_orchestrate with
 * that progress model, lowers it with megacu/runtime/co_resident.h (GEMM
 * tiles, then one allreduce unit per event slot waiting for that slot on
 * every PE) and runs it as ONE cooperative persistent launch of the generic
 * device loop. Same arguments, buffers, results and event tensor as
 * megacu_cuda_gemm_allreduce_phased_f32, plus `control`: device memory of
 * megacu_b200_co_resident_control_bytes() bytes (the graph and the queue
 * counters, rewritten by every call; one per concurrent call). A wait that
 * gave up is reported by megacu_b200_co_resident_status (detail 40; info[0]
 * node, info[1] tile). Lowering errors keep megacu's status convention
 * (unsupported/8-10, invalid_argument/2 and /6; see co_resident.h).
 */
megacu_status megacu_cuda_gemm_allreduce_f32_co_resident(
    megacu_driver_view driver, const float *a, const float *b, float *partial,
    float *out, void *events, void *control, megacu_gemm_ar_problem problem);
megacu_status megacu_b200_co_resident_control_bytes(int64_t *bytes);
megacu_status megacu_b200_co_resident_status(void *control, void *stream, int64_t info[2]);

/*
 * Allocation-free single-PE form of megacu_cuda_gemm_allreduce_bf16 (no
 * counterpart in megacu). For callers that cannot allocate device memory for
 * the kernel's scratch: plugin hosts that pass an operator only its inputs
 * and outputs, processes whose device memory belongs to another allocator,
 * and latency-critical loops that must not call cudaMalloc. The caller still
 * passes a, b and out; the scratch (task-queue control block and event
 * tensor) lives in a 256 KiB array built into the library, one per GPU, held
 * until the process exits. Limits: team_n_pes must be 1 (unsupported/51);
 * at most 8183 output tiles (invalid_argument/52). Every call on a GPU shares
 * that array, so calls that overlap on the GPU race — issue them in stream
 * order. Each call clears the array's queue tickets and error word first,
 * so an error is reported for the call that met it and never stops a later
 * call. The first call on a device (and the first after its context was
 * reset) looks up the array's address with that device current; make it
 * before any stream capture.
 */
megacu_status megacu_cuda_gemm_bf16_noalloc(megacu_driver_view driver,
                                            const void *a, const void *b,
                                            void *out,
                                            megacu_gemm_ar_problem_v2 problem);

/*
 * Device address (*events) and size (*bytes, may be NULL) of `device`'s
 * built-in scratch used by megacu_cuda_gemm_bf16_noalloc (no counterpart in
 * megacu). Allocates nothing. Pass the address to megacu_b200_events_status
 * for the last call's error (read and cleared) and to
 * megacu_b200_events_counters for completion counters summed over every
 * allocation-free call on that GPU (counters[7] counts every error).
 */
megacu_status megacu_b200_noalloc_scratch(int32_t device, void **events, int64_t *bytes);

/* Bytes of workspace / events a bf16 call needs for `problem` on n_pes PEs. */
megacu_status megacu_b200_workspace_bytes(megacu_gemm_ar_problem_v2 problem,
                                          int32_t n_pes, int64_t *bytes);
megacu_status megacu_b200_events_bytes(megacu_gemm_ar_problem_v2 problem,
                                       int32_t n_pes, int64_t *bytes);

/*
 * Tile plan of a bf16 call (host only, no GPU): info[0] tile_m, [1] tile_n,
 * [2] m_tiles, [3] n_tiles, [4] one_shot, [5] partial slots per parity plane,
 * [6] raster band height in tile rows, [7] bytes per element on the wire,
 * [8] 1 if 2-CTA clusters compute 256-row pair tiles (enum megacu_cta_pairs),
 * [9] GEMM tickets per call (tiles, or pair tiles).
 */
megacu_status megacu_b200_plan_info(megacu_gemm_ar_problem_v2 problem,
                                    int32_t n_pes, int32_t info[10]);

/*
 * Where the device task queue sends raster index r (host only): out[0] tile
 * row, out[1] tile column, out[2] owner PE, out[3] index among the owner's
 * tiles. Tile id = out[0] * n_tiles + out[1]. For MEGACU_MODE_ALLGATHER the
 * raster depends on the PE (each starts with its own shard): out[2] is the
 * PE whose shard holds the tile's rows, out[3] the index within that shard;
 * megacu_b200_plan_tile answers for PE 0, megacu_b200_plan_tile_on for any.
 */
megacu_status megacu_b200_plan_tile(megacu_gemm_ar_problem_v2 problem,
                                    int32_t n_pes, int32_t r, int32_t out[4]);
megacu_status megacu_b200_plan_tile_on(megacu_gemm_ar_problem_v2 problem,
                                       int32_t n_pes, int32_t my_pe, int32_t r,
                                       int32_t out[4]);

/*
 * Where a CTA pair's GEMM ticket q goes (host only; plans with pairs):
 * out[0], out[1] = raster indices of the upper and lower 128-row tiles the
 * two CTAs of the cluster compute (pass them to megacu_b200_plan_tile).
 * MEGACU_UNSUPPORTED (detail 27) if the plan computes no CTA pairs.
 */
megacu_status megacu_b200_plan_pair(megacu_gemm_ar_problem_v2 problem,
                                    int32_t n_pes, int32_t q, int32_t out[2]);

/*
 * Reads the device status word of `events` after the stream has finished
 * (synchronises the stream). code MEGACU_OK if the last calls completed;
 * MEGACU_BACKEND_ERROR with detail 40 if a cross-GPU wait timed out
 * (info[0] = tile, info[1] = peer PE, info[2] = which wait), 41 if a local
 * pipeline wait timed out and 42 if a bounds check of the checked build
 * failed; info[3] = the detail. The word is cleared by the call.
 * Which wait (info[2]):
 *   fused GEMM + exchange kernel: 1 producer's task ring, 2 producer's free
 *     stage, 3 MMA's task ring, 4 MMA's free accumulator, 5 MMA's full stage,
 *     6 epilogue's task ring, 7 epilogue's full accumulator, 8 a PE's partial
 *     flag (exchange), 9 a PE's done flag (two-shot completion);
 *   all-gather: 21 a peer's shard-ready flag, 22 a peer's shard-copied flag,
 *     23 the GEMM producer's wait for copied rows;
 *   single-launch MLP chain: 11 producer's task ring, 12 a dependency
 *     counter (act_ready / x_ready), 13 producer's free stage, 14-16 MMA's
 *     task ring / free accumulator / full stage, 17 epilogue's task ring,
 *     19 epilogue's full accumulator, 18 a PE's partial flag, 20 the final
 *     wait for the last block's rows;
 *   checked build: 30 all-gather copy chunk, 31 all-gather A row, 32 chain
 *     exchange indices, 34 chain publish indices, 35 chain dependency index.
 */
megacu_status megacu_b200_events_status(void *events, void *stream,
                                        int64_t info[4]);

/*
 * Cumulative device counters kept in `events` (task and event completions):
 * counters[0] GEMM tile tasks, [1] reduce tasks, [2] partial publishes,
 * [3] partial acquires, [4] final-tile publishes, [5] final-tile acquires,
 * [6] launches. Synchronises the stream.
 */
megacu_status megacu_b200_events_counters(void *events, void *stream,
                                          uint64_t counters[8]);

/* ---- team: symmetric heap over NVLink peer mappings ---------------------- */

/* Size of the opaque handle a PE exports for its heap. */
#define MEGACU_B200_TEAM_HANDLE_BYTES 128

/*
 * Creates this PE's team object and its symmetric heap (one cudaMalloc of
 * heap_bytes on `device`, zero-filled). Replaces nvshmem_init + the
 * symmetric heap of megacu's NVSHMEM backend (backends/nvshmem.h:19-38).
 */
megacu_status megacu_b200_team_create(int32_t my_pe, int32_t n_pes,
                                      int32_t device, int64_t heap_bytes,
                                      void **team);
/* Writes this PE's heap handle (MEGACU_B200_TEAM_HANDLE_BYTES bytes). */
megacu_status megacu_b200_team_export(void *team, void *handle);
/* Maps every peer's heap; handles = n_pes handles in PE order. */
megacu_status megacu_b200_team_connect(void *team, const void *handles);
/*
 * Bump-allocates `bytes` (256-byte aligned) from the symmetric heap. Every PE
 * must make the same sequence of calls, as with nvshmem_malloc.
 */
megacu_status megacu_b200_team_malloc(void *team, int64_t bytes, void **ptr);
megacu_status megacu_b200_team_info(void *team, int32_t *my_pe,
                                    int32_t *n_pes, void **heap_base,
                                    int64_t *heap_bytes);
/*
 * Enqueues a team-wide barrier on `stream` (a one-warp kernel over the peer
 * flags; bounded). Replaces nvshmem_barrier_all at megacu's call sites
 * (megacu_gemm_allreduce_phased.cu:186-193) without a host synchronisation.
 */
megacu_status megacu_b200_team_barrier(void *team, void *stream);
/* Collective when the team has a multicast region (see below). */
megacu_status megacu_b200_team_destroy(void *team);

/*
 * Launch adapter for processes on one node (a B200 addition; megacu relies on
 * NVSHMEM's launcher and lists MPI / torch adapters as future work): every
 * PE calls with the same `session` (1-64 characters, unique per team, the
 * role of an NVSHMEM unique id) and its own `bytes`-byte blob; `all`
 * receives n_pes * bytes, every PE's blob in PE order. Runs over an abstract
 * unix socket served by PE 0 (so the PEs share a network namespace), bounded
 * by timeout_ms: a PE that does not join, joins twice or sends another size
 * makes the PEs that notice it return MEGACU_BACKEND_ERROR / 39. Host only,
 * no GPU needed.
 */
megacu_status megacu_b200_exchange_local(const char *session, int32_t my_pe, int32_t n_pes,
                                         const void *mine, int64_t bytes, void *all,
                                         int64_t timeout_ms);
/* megacu_b200_team_create + _export + megacu_b200_exchange_local + _connect,
 * collective: a connected team in one call. */
megacu_status megacu_b200_team_create_local(const char *session, int32_t my_pe,
                                            int32_t n_pes, int32_t device,
                                            int64_t heap_bytes, int64_t timeout_ms,
                                            void **team);

/*
 * Optional multicast (NVLS) region of a connected team, one process per PE:
 * each PE's own device memory bound to one NVSwitch multicast object, so the
 * two-shot allreduce can reduce partials in the switch (multimem.ld_reduce)
 * and store each sum into every PE at once (multimem.st). Collective set-up:
 *   megacu_b200_team_multicast_export(team, bytes, mine)   every PE
 *   exchange the MEGACU_B200_TEAM_HANDLE_BYTES blobs, PE order
 *   megacu_b200_team_multicast_connect(team, all)          every PE
 * `bytes` is rounded up to the multicast granularity (512 MiB on B200).
 * PE 0 hands the object to the others over an abstract unix socket named in
 * its blob. MEGACU_UNSUPPORTED (detail 35) when the device, driver or team
 * shape (one PE, or PEs sharing a process) cannot have one; callers then use
 * the heap alone. megacu_b200_team_multicast_malloc is the region's
 * symmetric allocator (same order on every PE). Workspace and out of a
 * two-shot bf16 allreduce placed here select the in-switch reduction.
 */
megacu_status megacu_b200_team_multicast_export(void *team, int64_t bytes, void *handle);
megacu_status megacu_b200_team_multicast_connect(void *team, const void *handles);
megacu_status megacu_b200_team_multicast_malloc(void *team, int64_t bytes, void **ptr);
/* base = NULL and bytes = 0 when the team has no multicast region. */
megacu_status megacu_b200_team_multicast_info(void *team, void **base, int64_t *bytes);

/* ---- component link anchors (last line of each megacu component source) -- */

int megacu_dispatcher_explicit_attrs_component(void);
int megacu_scheduler_explicit_asap_component(void);
int megacu_platform_cuda_component(void);
int megacu_backend_nvshmem_component(void);
int megacu_target_runtime_component(void);

/* Library version string. */
const char *megacu_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MEGACU_B200_H_ */
