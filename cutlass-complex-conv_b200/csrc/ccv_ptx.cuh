// Thin inline-PTX wrappers for the sm_100a features the complex-conv kernels
// use: mbarriers, TMA tensor loads, tcgen05 MMA / TMEM, and a bounded wait.
//
// Every wait on an mbarrier goes through `mbar_wait_bounded`: it gives up
// after CCV_WAIT_TIMEOUT_NS of wall time (read from %globaltimer), records an
// error code in a device status word and returns false, so a mistake in a
// transaction count can never spin a GPU forever.
#pragma once

#include <cuda.h>
#include <cstdint>

#ifndef CCV_WAIT_TIMEOUT_NS
#define CCV_WAIT_TIMEOUT_NS 1000000000ull  // 1 s for any single barrier wait
#endif

namespace ccv {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred));
  return pred;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with cluster-scope acquire: orders the waiter after writes that
// other CTAs of the cluster released with mbarrier.arrive.release.cluster.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Makes this thread's generic-proxy shared-memory writes visible to the
// async proxy (TMA, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Records a failed wait: `code` into *status (first error wins) and, with
// MIRROR, into the host-mapped mirror whose device address the library's
// status block keeps in its words 2-3 (status points at word 0 of that
// block), so host code sees the timeout without synchronizing.
template <bool MIRROR = true>
__device__ __forceinline__ void report_status(int* status, int code) {
  if (status == nullptr) return;
  atomicCAS(status, 0, code);
  if constexpr (MIRROR) {
    int* host = *reinterpret_cast<int* const volatile*>(status + 2);
    if (host != nullptr) {
      *reinterpret_cast<volatile int*>(host) = code;
      __threadfence_system();
    }
  }
}

// Wait for the phase with the given parity to complete, for at most
// CCV_WAIT_TIMEOUT_NS.  On timeout, reports `code` (report_status) and
// returns false.
template <bool CLUSTER_ACQUIRE = false, bool MIRROR = true>
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int* status,
                                                  int code) {
  auto test = [&]() {
    return CLUSTER_ACQUIRE ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  };
#pragma unroll 1
  for (int i = 0; i < 256; ++i) {
    if (test()) return true;
  }
  const uint64_t t0 = globaltimer();
#pragma unroll 1
  while (true) {
    if (test()) return true;
    if (globaltimer() - t0 > CCV_WAIT_TIMEOUT_NS) {
      report_status<MIRROR>(status, code);
      return false;
    }
  }
}

// Same bound, for warps off the critical path (epilogue, converters): after
// a short poll they sleep between tests, leaving issue slots to the
// single-thread TMA producer and MMA issuer warps of the same SM.
template <bool CLUSTER_ACQUIRE = false>
__device__ __forceinline__ bool mbar_wait_bounded_backoff(uint32_t bar, uint32_t parity,
                                                          int* status, int code) {
  auto test = [&]() {
    return CLUSTER_ACQUIRE ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  };
#pragma unroll 1
  for (int i = 0; i < 8; ++i) {
    if (test()) return true;
  }
  const uint64_t t0 = globaltimer();
  uint32_t ns = 32;
#pragma unroll 1
  while (true) {
    if (test()) return true;
    if (globaltimer() - t0 > CCV_WAIT_TIMEOUT_NS) {
      report_status(status, code);
      return false;
    }
    asm volatile("nanosleep.u32 %0;" ::"r"(ns));
    if (ns < 256) ns <<= 1;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// Programmatic dependent launch: wait until the grids this launch depends on
// have completed and their memory is visible (returns at once without PDL),
// then allow the next PDL launch on the stream to begin its prologue.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// TMA tile stores shared -> global (bulk-group completion).  Elements of the
// box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until the issuing thread's committed bulk stores have read their
// shared-memory source (the buffer may be rewritten).
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Same, allowing the most recent bulk group to still be reading.
__device__ __forceinline__ void bulk_wait_read_le1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Wait until the issuing thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completing `bytes` on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Orders this thread's generic-proxy memory accesses before its later
// async-proxy ones (bulk copies), in every state space.
__device__ __forceinline__ void fence_proxy_async_all() {
  asm volatile("fence.proxy.async;" ::: "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Asks for one box of a tensor to be brought into L2 (no shared-memory
// destination, no completion to wait for).  A performance hint only: L2 is
// the point of coherence, so issuing it before griddepcontrol.wait cannot
// return stale data to a later load.
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2,
                                                   int c3) {
  asm volatile(
      "cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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

// D[tmem] (+)= A[smem] * B[smem]^T, TF32 inputs, FP32 accumulate.
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued MMAs of this thread finish.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// Pins registers that an asynchronous tcgen05.ld wrote: an empty volatile asm
// that reads and redefines each one, placed after tcgen05.wait::ld, so no use
// of them can be scheduled before the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// lane (base_lane + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7])
      : "r"(taddr));
}

// Width-generic form (W = 8, 16 or 32).
template <int W>
__device__ __forceinline__ void tmem_ld_32x32b(uint32_t taddr, uint32_t (&v)[W]) {
  if constexpr (W == 32) {
    tmem_ld_32x32b_x32(taddr, v);
  } else if constexpr (W == 16) {
    tmem_ld_32x32b_x16(taddr, v);
  } else {
    static_assert(W == 8, "8, 16 or 32 columns");
    tmem_ld_32x32b_x8(taddr, v);
  }
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor for a K-major operand stored in the 64-byte
// swizzle layout: rows of 64 bytes (16 fp32 along K), 8-row groups 512 bytes
// apart.  `smem_addr` may be advanced by 32 bytes to address the second
// 8-element K step inside the 64-byte row.
__device__ __forceinline__ uint64_t desc_kmajor_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);           // start address
  d |= static_cast<uint64_t>(1u) << 16;                              // LBO (unused, swizzled K-major)
  d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;           // SBO: 8 rows x 64 B
  d |= static_cast<uint64_t>(1u) << 46;                              // descriptor version (sm_100)
  d |= static_cast<uint64_t>(4u) << 61;                              // layout: SWIZZLE_64B
  return d;
}

// Same for the 128-byte swizzle layout: rows of 128 bytes (32 fp32 along K),
// 8-row groups 1024 bytes apart; advance by 32 bytes per 8-element K step.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>((1024u >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;                              // layout: SWIZZLE_128B
  return d;
}

// ---------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// 16-byte load from shared memory of a CTA of the cluster (address from mapa).
// (No "memory" clobber: callers order these reads with cluster barriers, and
// leaving them unordered lets several remote loads be in flight at once.)
__device__ __forceinline__ float4 ld_shared_cluster_v4(uint32_t addr) {
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "r"(addr));
  return v;
}

// Cluster-wide barrier.  The non-.aligned forms count threads, so a warp
// whose lanes arrive at different times (one lane ran a role loop alone) is
// still waited for in full.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\t"
               "barrier.cluster.wait.acquire;" ::: "memory");
}

// CTA-wide barrier that counts threads, not warps.  __syncthreads() is the
// .aligned form, which PTX leaves undefined unless every lane of a warp
// reaches it together; after a branch that one lane runs alone (a producer or
// MMA loop, a bulk wait) the other lanes get there first.  The compiler's
// reconvergence made the aligned form wait in a B200 test (a lane held 2 us
// before the barrier; every thread read its flag after it), but only this
// form is defined there, so every barrier that follows such a branch is it.
__device__ __forceinline__ void cta_sync() { asm volatile("barrier.sync 0;" ::: "memory"); }

// cta_sync() that also returns whether `v` was true in any thread.
__device__ __forceinline__ bool cta_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.or.pred q, 0, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

// Arrive on an mbarrier that may live in another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Arrival without release semantics, for "accumulator buffer free" signals:
// the epilogue's tcgen05.ld reads are complete once tcgen05.wait::ld returns,
// and nothing else the arriving thread wrote is read by the waiter.  A
// release arrival would first wait for the thread's earlier memory
// operations - the TMA stores it just issued included - which measured
// ~2.8k cycles per tile in the pair kernels' epilogue.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// 32-bit store to shared memory of a CTA of the cluster (cluster address).
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void nanosleep(uint32_t ns) {
  asm volatile("nanosleep.u32 %0;" ::"r"(ns));
}

// TMA tile load by one CTA of a pair; completion (bytes) is signalled on the
// mbarrier at `bar_cluster` (a shared::cluster address, possibly in the peer).
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int c0, int c1, int c2,
                                                 int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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

// Pair MMA (issued by the even CTA): A rows from both CTAs (M = 256), B
// columns split across the CTAs (N/2 each), D rows land in each CTA's TMEM.
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at the same offset in both CTAs of the pair once the
// pair MMAs issued so far complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

// Instruction descriptor for kind::tf32, FP32 accumulator, K-major A and B.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t m, uint32_t n, bool negate_b) {
  return (1u << 4)                        // D format: F32
         | (2u << 7)                      // A format: TF32
         | (2u << 10)                     // B format: TF32
         | ((negate_b ? 1u : 0u) << 14)   // negate B
         | ((n >> 3) << 17)               // N / 8
         | ((m >> 4) << 24);              // M / 16
}

}  // namespace ptx
}  // namespace ccv
