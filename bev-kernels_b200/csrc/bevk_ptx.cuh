// bevk_ptx.cuh -- inline-PTX wrappers for sm_100a: mbarriers, TMA tile loads,
// tcgen05 (TMEM allocation, UMMA issue, commit, TMEM loads) and the bounded
// waits every barrier spin in this library goes through.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace bevk {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- dependent launch
// Programmatic dependent launch.  launch_dependents lets the stream's next
// kernel (launched with cudaLaunchAttributeProgrammaticStreamSerialization)
// place its CTAs once every CTA of this grid has issued it or exited;
// wait_prerequisites blocks until the previous kernel of the stream has
// completed and its memory writes are visible.  Both are no-ops in a launch
// without that attribute.  A kernel reads or writes no global memory that
// another kernel may touch before its wait.
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_wait_prerequisites() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Watchdog limit for any barrier wait: far above any legitimate stall of these
// kernels (microseconds), far below a hung-GPU timeout.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Bounded wait on phase `parity` of `bar`.  Returns false (after recording
// `site` in *err_word and raising *abort_flag) when `limit_ns` expires or when
// another role of the same CTA already aborted.  The clock and the abort flag
// are read on every 256th retry; try_wait itself suspends the thread for a
// hardware-defined interval, so a limit shorter than the default is also
// checked on the first retry (otherwise a short wait could finish before the
// limit is ever looked at).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int *abort_flag,
                                                  unsigned int *err_word,
                                                  unsigned int site,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u || (it == 1u && limit_ns < kWaitLimitNs)) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(err_word, 0u, site);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Device-scope exchange / release store / acquire load of 64-bit words in
// global memory (CTAs of one grid meeting on a ticket), and the grid's
// temporal launch number (distinct for every launch in a context).
__device__ __forceinline__ unsigned long long atom_exch_acq_rel_gpu(unsigned long long *p,
                                                                    unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.exch.b64 %0, [%1], %2;"
               : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release_gpu(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// 16-bit read-only load, issued where it stands (volatile: the compiler keeps
// a batch of them ahead of the code that uses the values).
__device__ __forceinline__ uint16_t ld_global_nc_u16(const void *p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void prefetch_l1(const void *p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
__device__ __forceinline__ unsigned long long grid_id() {
  unsigned long long g;
  asm volatile("mov.u64 %0, %%gridid;" : "=l"(g));
  return g;
}

// Cluster-scope variants (paired-CTA kernels): a wait that must observe
// arrivals released by the other CTA of the cluster.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint32_t bar, uint32_t parity,
                                                          volatile int *abort_flag,
                                                          unsigned int *err_word,
                                                          unsigned int site,
                                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 0u || (it == 1u && limit_ns < kWaitLimitNs)) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(err_word, 0u, site);
        *abort_flag = 1;
        return false;
      }
    }
  }
}
// Arrive on an mbarrier given by its shared::cluster address, possibly in the
// other CTA of the cluster (default release semantics, as CUTLASS's cluster
// barriers use).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// Whole-cluster execution barrier (all threads of both CTAs), release/acquire.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ---------------------------------------------------------------- proxies
// Orders this thread's generic-proxy shared-memory writes before subsequent
// async-proxy reads (tcgen05.mma operands written with st.shared).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
// 2-D tiled bulk-tensor load into this CTA's shared memory, completing on
// `bar` (transaction bytes).  c0 is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, uint32_t bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// Paired-CTA tile load: the copy lands in this CTA's shared memory and its
// completion bytes are counted on `bar`, which may be the leader CTA's barrier
// (shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void *tmap, uint32_t bar,
                                                 int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// canonical 128-byte-swizzled layout: 128-byte rows, 8-row (1024-byte) swizzle
// atoms stacked along M/N.  Fields: start address >> 4 (bits 0-13), leading
// byte offset >> 4 (16-29; unused for swizzled K-major, set to 1), stride
// byte offset >> 4 (32-45; 1024 B between 8-row groups), descriptor version 1
// (46-47), base offset 0 (49-51, tiles are 1024-byte aligned), layout type
// SWIZZLE_128B = 2 (61-63).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16 with fp32 accumulation,
// both operands K-major.  ab_fmt: 0 = f16, 1 = bf16.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t ab_fmt, uint32_t m, uint32_t n) {
  return (1u << 4)              // D format: f32
         | (ab_fmt << 7)        // A format
         | (ab_fmt << 10)       // B format
         | ((n >> 3) << 17)     // N / 8
         | ((m >> 4) << 24);    // M / 16
}

// D[tmem] (+)= A[smem] * B[smem]^T, single CTA, issued by one thread.
__device__ __forceinline__ void umma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// As umma_commit, arriving on the barrier at offset `bar` in every CTA of
// `cta_mask` of the cluster.
__device__ __forceinline__ void umma_commit_multicast(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// this CTA's shared memory to shared memory of a CTA of the cluster; the copy
// completes its bytes as transactions on the mbarrier `bar` (a shared::cluster
// address in the destination CTA).  Source data written with st.shared must be
// ordered before the copy with fence_proxy_async_smem().
__device__ __forceinline__ void bulk_copy_smem_to_cluster(uint32_t dst_cluster, uint32_t src_cta,
                                                          uint32_t bytes, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

// Paired-CTA (cta_group::2) forms: TMEM allocation shared by the two CTAs of
// a cluster (same warp in each CTA), M=256 MMA issued by the leader CTA, and
// its completion signalled to the barrier at the same offset in both CTAs.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the barrier at offset `bar` in every CTA of `cta_mask` when
// the MMAs issued so far by this thread have completed (a commit, not a copy).
__device__ __forceinline__ void umma_commit_pair_both(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns (this warp's lane quadrant).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
template <int N>
__device__ __forceinline__ void tmem_ld_32x32b(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(N == 16 || N == 32, "32x32b loads of 16 or 32 columns");
  if constexpr (N == 32) tmem_ld_32x32b_x32(taddr, r);
  else tmem_ld_32x32b_x16(taddr, r);
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 16-byte read-only global load issued only when `pred` != 0 (zeros otherwise);
// predication instead of a branch lets a thread keep many such loads in flight.
__device__ __forceinline__ uint4 ld_global_nc_v4_pred(const void *p, uint32_t pred) {
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %4, 0;\n\t"
      "@q ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%5];\n\t}"
      : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
      : "r"(pred), "l"(p));
  return v;
}

// N 32-bit words held in registers (N = 4: 16 bytes, N = 8: 32 bytes).
template <int N>
struct Words {
  uint32_t w[N];
};

// Unconditional read-only global vector load of 16 or 32 bytes (the address
// must be aligned to the size).  The 32-byte form is the sm_100 256-bit load.
template <int N>
__device__ __forceinline__ Words<N> ld_global_nc_words(const void *p) {
  Words<N> v;
  if constexpr (N == 4) {
    asm volatile("ld.global.nc.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(p));
  } else {
    static_assert(N == 8, "16- or 32-byte loads");
    asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]),
                   "=r"(v.w[5]), "=r"(v.w[6]), "=r"(v.w[7])
                 : "l"(p));
  }
  return v;
}

// As ld_global_nc_v4_pred, in the Words<4> form.
__device__ __forceinline__ Words<4> ld_global_nc_words4_pred(const void *p, uint32_t pred) {
  const uint4 v = ld_global_nc_v4_pred(p, pred);
  return Words<4>{{v.x, v.y, v.z, v.w}};
}

// Scheduling fence on registers: no instruction is emitted, but code using
// `v` afterwards cannot be hoisted above this point (nor above the volatile
// loads issued before it).  Used to keep a prefetch ahead of the arithmetic
// that consumes the previous batch.
__device__ __forceinline__ void reg_fence(uint4 &v) {
  asm volatile("" : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w));
}
__device__ __forceinline__ void reg_fence(uint2 &v) { asm volatile("" : "+r"(v.x), "+r"(v.y)); }
__device__ __forceinline__ void reg_fence(float &v) { asm volatile("" : "+f"(v)); }
template <int N>
__device__ __forceinline__ void reg_fence(Words<N> &v) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(v.w[i]));
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

}  // namespace ptx
}  // namespace bevk
