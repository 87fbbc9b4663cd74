// Thin inline-PTX layer for sm_100a: mbarriers, TMA tile loads, tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads) and system-scope flags.
//
// Every wait in here is bounded: it polls an abort word and `%globaltimer`
// and returns false instead of spinning forever, so no protocol bug or dead
// peer can hang the GPU.
//
// No load in this file uses cluster multicast: tiles are fetched per CTA.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace megacu_b200::ptx {

__device__ __forceinline__ std::uint32_t smem_addr(void const *p) {
  return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ std::uint64_t now_ns() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ std::uint32_t lane_id() {
  std::uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ---- plain global flags ----------------------------------------------------

__device__ __forceinline__ std::uint32_t ld_acquire_sys(std::uint32_t const *p) {
  std::uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ std::uint32_t ld_acquire_gpu(std::uint32_t const *p) {
  std::uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ std::uint32_t ld_relaxed_gpu(std::uint32_t const *p) {
  std::uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ std::uint32_t ld_relaxed_sys(std::uint32_t const *p) {
  std::uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(std::uint32_t *p, std::uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys(std::uint32_t *p, std::uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// Publishes a flag for data this thread (or its warp, after a __syncwarp)
// wrote into THIS GPU's own memory. The GPU-scope fence makes those writes
// visible at this GPU's L2, which is where every peer's NVLink load of that
// memory is served; the flag itself is a relaxed system-scope store. On a
// B200 under NVLink load a system-scope fence costs several microseconds per
// call (it orders against all of the SM's outstanding peer traffic), this
// costs none; readers acquire at system scope (wait_flag).
__device__ __forceinline__ void publish_local_data(std::uint32_t *flag, std::uint32_t v) {
  st_relaxed_sys(flag, v);
}

// Adds `v` to a counter (this GPU's or a peer's) with release semantics at
// system scope: the issuing thread's earlier writes are visible to whoever
// acquires the counter's new value.
__device__ __forceinline__ void red_release_sys_add(std::uint32_t *p, std::uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Adds `v` to a counter in this GPU's memory with release semantics at GPU
// scope (readers on this GPU only).
__device__ __forceinline__ void red_release_gpu_add(std::uint32_t *p, std::uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Orders this thread's earlier generic-proxy accesses (and the acquires that
// made other threads' writes visible to it) before its later async-proxy
// ones, e.g. TMA loads of data that other SMs or GPUs wrote.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- NVSwitch multicast (multimem) ----------------------------------------------
// `mc` must be an address in a multicast mapping (a team's multicast region).

// The sum over every PE's copy of 16 bytes (8 bf16) at `mc`, reduced in the
// switch with fp32 accumulation and rounded to bf16 once.
__device__ __forceinline__ uint4 multimem_ld_reduce_bf16x8(void const *mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

// Stores 16 bytes into every PE's copy at `mc`.
__device__ __forceinline__ void multimem_st_v4(void *mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};"
               :: "l"(mc), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Orders this thread's accesses made through one virtual mapping of a
// location (the multicast one) with those made through another (unicast).
__device__ __forceinline__ void fence_proxy_alias() {
  asm volatile("fence.proxy.alias;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(std::uint32_t id, std::uint32_t threads) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

// ---- vector global access ----------------------------------------------------

__device__ __forceinline__ uint4 ld_cg_v4(void const *p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4(void *p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ---- mbarrier ------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(std::uint64_t *bar, std::uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy accesses to shared memory (e.g.
// mbarrier.init) before its later async-proxy ones (TMA loads that complete
// on those barriers).
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(std::uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(std::uint64_t *bar, std::uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_test(std::uint32_t bar, std::uint32_t parity) {
  std::uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with `parity` of `bar` to complete. Gives up (returns
// false) when `*abort_word` (a global word; nullptr = never) becomes non-zero
// or `timeout_ns` elapses.
__device__ __forceinline__ bool mbar_wait(std::uint64_t *bar, std::uint32_t parity,
                                          std::uint32_t const *abort_word,
                                          std::uint64_t timeout_ns) {
  std::uint32_t const a = smem_addr(bar);
  if (mbar_test(a, parity)) {
    return true;
  }
  std::uint64_t const start = now_ns();
  for (std::uint32_t spin = 1;; ++spin) {
    if (mbar_test(a, parity)) {
      return true;
    }
    if ((spin & 127u) == 0) {
      if (abort_word != nullptr && ld_relaxed_gpu(abort_word) != 0) {
        return false;
      }
      if (now_ns() - start > timeout_ns) {
        return false;
      }
    }
  }
}

// ---- clusters (CTA pairs) --------------------------------------------------------

__device__ __forceinline__ std::uint32_t cluster_ctarank() {
  std::uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ std::uint32_t map_to_rank(void const *local, std::uint32_t rank) {
  std::uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(local)), "r"(rank));
  return out;
}

// Arrive once on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(std::uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
               :: "r"(cluster_addr) : "memory");
}

// Relaxed form, for pure events that publish no data of this thread. A
// release at cluster scope costs the issuing thread about a microsecond when
// it has TMA loads in flight (measured), so the per-k-block relay uses this.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(std::uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];"
               :: "r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void st_shared_remote(std::uint32_t cluster_addr, std::int32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" :: "r"(cluster_addr), "r"(v) : "memory");
}


// 16 bytes into the shared memory of a CTA of this cluster.
__device__ __forceinline__ void st_shared_remote_v4(std::uint32_t cluster_addr, std::uint32_t a,
                                                    std::uint32_t b, std::uint32_t c,
                                                    std::uint32_t d) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};"
               :: "r"(cluster_addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ bool mbar_test_cluster(std::uint32_t bar, std::uint32_t parity) {
  std::uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// mbar_wait for barriers that other CTAs of the cluster arrive on: the wait
// acquires at cluster scope.
__device__ __forceinline__ bool mbar_wait_cluster(std::uint64_t *bar, std::uint32_t parity,
                                                  std::uint32_t const *abort_word,
                                                  std::uint64_t timeout_ns) {
  std::uint32_t const a = smem_addr(bar);
  if (mbar_test_cluster(a, parity)) {
    return true;
  }
  std::uint64_t const start = now_ns();
  for (std::uint32_t spin = 1;; ++spin) {
    if (mbar_test_cluster(a, parity)) {
      return true;
    }
    if ((spin & 127u) == 0) {
      if (abort_word != nullptr && ld_relaxed_gpu(abort_word) != 0) {
        return false;
      }
      if (now_ns() - start > timeout_ns) {
        return false;
      }
    }
  }
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---- TMA -------------------------------------------------------------------------

__device__ __forceinline__ void prefetch_tensor_map(CUtensorMap const *map) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(map) : "memory");
}

// 2-D tile load global -> shared, completion counted on `bar` in bytes.
__device__ __forceinline__ void tma_load_2d(CUtensorMap const *map, std::uint64_t *bar,
                                            void *dst, std::int32_t x, std::int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      :: "r"(smem_addr(dst)), "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

// 2-D tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of the pair's leader CTA (`bar_cluster` from map_to_rank).
__device__ __forceinline__ void tma_load_2d_pair(CUtensorMap const *map, std::uint32_t bar_cluster,
                                                 void *dst, std::int32_t x, std::int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      :: "r"(smem_addr(dst)), "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// ---- tcgen05 / TMEM ---------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(std::uint32_t *dst, std::uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_addr(dst)), "r"(columns) : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(std::uint32_t taddr, std::uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               :: "r"(taddr), "r"(columns) : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16(std::uint32_t d_tmem, std::uint64_t a_desc,
                                         std::uint64_t b_desc, std::uint32_t idesc,
                                         std::uint32_t accumulate) {
  std::uint32_t const no_mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(no_mask)
      : "memory");
}

// ---- the CTA-pair (cta_group::2) forms: both CTAs of the pair allocate the
// same TMEM columns; the leader issues MMAs whose A and B halves and
// accumulator rows live in both CTAs.

__device__ __forceinline__ void tmem_alloc_pair(std::uint32_t *dst, std::uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_addr(dst)), "r"(columns) : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(std::uint32_t taddr, std::uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
               :: "r"(taddr), "r"(columns) : "memory");
}

__device__ __forceinline__ void umma_f16_pair(std::uint32_t d_tmem, std::uint64_t a_desc,
                                              std::uint64_t b_desc, std::uint32_t idesc,
                                              std::uint32_t accumulate) {
  std::uint32_t const no_mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, "
      "{%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(no_mask)
      : "memory");
}

// Arrives once on the leader's `bar` when every previously issued pair MMA of
// this thread has completed.
__device__ __forceinline__ void umma_commit_pair(std::uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_addr(bar)) : "memory");
}

// Arrives once on `bar` when every previously issued tcgen05.mma of this
// thread has completed.
__device__ __forceinline__ void umma_commit(std::uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_addr(bar)) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i receives lane
// (base_lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_load_32x32b_x32(std::uint32_t taddr, std::uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_load() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- UMMA descriptors ---------------------------------------------------------------

// Shared-memory matrix descriptor (sm100 format, "version" 1):
// [0,14) start >> 4, [16,30) leading byte offset >> 4, [32,46) stride byte
// offset >> 4, [46,48) version = 1, [61,64) layout (2 = 128-byte swizzle).
__device__ __forceinline__ std::uint64_t smem_desc_sw128(std::uint32_t start,
                                                         std::uint32_t lbo_bytes,
                                                         std::uint32_t sbo_bytes) {
  std::uint64_t d = 0;
  d |= static_cast<std::uint64_t>((start >> 4) & 0x3fffu);
  d |= static_cast<std::uint64_t>((lbo_bytes >> 4) & 0x3fffu) << 16;
  d |= static_cast<std::uint64_t>((sbo_bytes >> 4) & 0x3fffu) << 32;
  d |= static_cast<std::uint64_t>(1) << 46;
  d |= static_cast<std::uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B,
// A K-major, B MN-major (row-major [K, N] operand), shape M x N.
__host__ __device__ constexpr std::uint32_t idesc_bf16_f32(std::uint32_t m, std::uint32_t n,
                                                           bool b_mn_major) {
  return (1u << 4)                       // D format: f32
         | (1u << 7)                     // A format: bf16
         | (1u << 10)                    // B format: bf16
         | (0u << 15)                    // A major: K
         | ((b_mn_major ? 1u : 0u) << 16)  // B major
         | ((n >> 3) << 17)              // N / 8
         | ((m >> 4) << 24);             // M / 16
}

// ---- conversions ----------------------------------------------------------------------

__device__ __forceinline__ std::uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<std::uint32_t *>(&v);
}

__device__ __forceinline__ float bf16_lo(std::uint32_t v) {
  return __uint_as_float(v << 16);
}

__device__ __forceinline__ float bf16_hi(std::uint32_t v) {
  return __uint_as_float(v & 0xffff0000u);
}

}  // namespace megacu_b200::ptx
