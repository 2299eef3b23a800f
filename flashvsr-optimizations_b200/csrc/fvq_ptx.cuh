// fvq_ptx.cuh -- inline-PTX wrappers for sm_100a: mbarriers, TMA / bulk copies,
// tcgen05 (TMEM alloc, block-scaled MMA, smem->TMEM copy, TMEM loads) and the
// FP8/FP4 conversions the quantizer uses.  Written from the PTX ISA; every
// wait is bounded in wall time (kDefaultWaitLimit, kErrWait* in fvq_internal.h).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace fvq {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// try_wait suspends the thread until the phase completes or for at most
// `hint_ns` (the hardware may return earlier); a completed phase wakes it at once.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity,
                                                   uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Suspend hint for a wait bounded by `limit_ns`: never longer than the limit,
// so a short limit is honoured however fast the awaited work is.
__device__ __forceinline__ uint32_t wait_hint_ns(uint64_t limit_ns) {
  return limit_ns < (1u << 20) ? static_cast<uint32_t>(limit_ns) : (1u << 20);
}

// Non-blocking: has the phase with `parity` completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Limits shorter than this are below what %globaltimer resolves (and try_wait
// may sleep longer than its hint): such a wait is one non-blocking test.
constexpr uint64_t kTimerResolutionNs = 1000;

// Wait until the phase with `parity` completes, for at most `limit_ns`
// nanoseconds of wall time (plus at most one suspend hint).  Returns false on
// timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  if (limit_ns < kTimerResolutionNs) return mbar_test_wait(bar, parity);
  const uint32_t hint = wait_hint_ns(limit_ns);
  if (mbar_try_wait_hint(bar, parity, hint)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_hint(bar, parity, hint)) return true;
    if (global_timer_ns() - start > limit_ns) return false;
  }
}

// ---------------------------------------------------------------- warp-uniform issue
// tcgen05 and TMA instructions take their operands from the warp's uniform
// registers.  Issuing them from one lane of a diverged branch moves every
// operand there instruction by instruction (measured: ~300 cycles per 4-MMA K
// step); the issuing warps therefore run their loops converged, wait in every
// lane, and let one elected lane issue.
__device__ __forceinline__ bool elect_one() {
  uint32_t p;
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, e;\n\t}"
      : "=r"(p));
  return p != 0;
}

// Warp index the compiler can see is uniform across the warp.
__device__ __forceinline__ int warp_index_uniform() {
  return __shfl_sync(0xFFFFFFFFu, static_cast<int>(threadIdx.x >> 5), 0);
}

// mbar_wait_bounded by every lane of a converged warp; lane 0's outcome for all.
__device__ __forceinline__ bool warp_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  const bool ok = mbar_wait_bounded(bar, parity, limit_ns);
  return __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
}

// ---------------------------------------------------------------- TMA / bulk copy
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- CTA pairs (clusters of 2)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// All threads of both CTAs.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// Arrive on an mbarrier of any CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_try_wait_cluster_hint(uint64_t* bar, uint32_t parity,
                                                           uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Bounded wait on a local mbarrier that other CTAs of the cluster arrive on.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity,
                                                          uint64_t limit_ns) {
  if (limit_ns < kTimerResolutionNs) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
  }
  const uint32_t hint = wait_hint_ns(limit_ns);
  if (mbar_try_wait_cluster_hint(bar, parity, hint)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait_cluster_hint(bar, parity, hint)) {
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// mbar_wait_cluster_bounded by every lane of a converged warp; lane 0's outcome for all.
__device__ __forceinline__ bool warp_wait_cluster_bounded(uint64_t* bar, uint32_t parity,
                                                          uint64_t limit_ns) {
  const bool ok = mbar_wait_cluster_bounded(bar, parity, limit_ns);
  return __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_dst)),
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

// Scale copies issued by the pair's even CTA: each CTA's shared memory at the
// descriptor's offset goes to the same TMEM address of that CTA.
__device__ __forceinline__ void tmem_cp_32x128b_x4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

__device__ __forceinline__ void tmem_cp_128x256b_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// M = 256 across the pair: each CTA supplies its 128 rows of A and half of
// the N columns of B at the descriptors' offsets; D rows are split likewise.
__device__ __forceinline__ void mma_nvf4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X"
      " [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Arrive on the mbarrier at `cluster_addr` (this CTA's or the peer's) once all
// tcgen05 operations issued so far by this thread complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          cluster_addr)
      : "memory");
}

// Tiled tensor loads into this CTA's shared memory whose completion is counted
// on an mbarrier of the pair's even CTA (`bar_cluster`, a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap,
                                                 uint32_t bar_cluster, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const void* tmap,
                                                 uint32_t bar_cluster, int32_t c0, int32_t c1,
                                                 int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Tiled tensor store shared -> global through a tensor map, tracked by the
// issuing thread's bulk groups.  Rows and columns past the map's extent are
// not written.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int32_t c0,
                                             int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// The shared-memory sources of this thread's committed bulk stores have been read.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// This thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_dst)),
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

// Block-scaled NVFP4 MMA, M=128 (one CTA), 16-element E4M3 scale blocks.
__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X"
      " [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// D (+)= A * B^T with E4M3 (or other 8/6/4-bit) operands named by `idesc`,
// no block scales; K = 32 per instruction.
__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Copy 32 rows x 16 bytes from shared memory into TMEM lanes 0-31, replicated
// to the four 32-lane sub-partitions (4 columns of 32 bits).
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// Arrive on `bar` once all tcgen05 operations issued so far by this thread complete.
// 128 TMEM lanes x 256 bits: lane i gets row i of the shared-memory source
// (two 16-byte core-matrix columns, LBO apart), columns [col, col+8).
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 columns of 32-bit values: thread i of the warp gets lane
// (base lane + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"):
//   [0,14) start>>4, [16,30) leading byte offset>>4, [32,46) stride byte offset>>4,
//   [46,48) version = 1, [49,52) base offset, [61,64) layout (0 none, 2 = 128B swizzle).
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 0x7) << 61;
  return d;
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with cudaLaunchAttributeProgrammaticStreamSerialization may start
// while the kernel before it in the stream is still finishing; grid_dependency_wait()
// returns once that kernel has completed and its memory operations are visible, so every
// thread waits before it touches global memory the previous kernel may write or read.
// grid_launch_dependents() lets the next such kernel start launching once every CTA of
// this grid has called it (or exited).
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- numerics
__device__ __forceinline__ float rcp_approx_ftz(float a) {
  float b;
  asm volatile("rcp.approx.ftz.f32 %0, %1;" : "=f"(b) : "f"(a));
  return b;
}

__device__ __forceinline__ float mul_ftz(float a, float b) {
  float c;
  asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(c) : "f"(a), "f"(b));
  return c;
}

// float -> E4M3 byte, round to nearest even, saturating.
__device__ __forceinline__ uint32_t f32_to_e4m3(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return r & 0xFFu;
}

// E4M3 byte -> float (exact, via f16).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  uint32_t h2;
  uint16_t in = static_cast<uint16_t>(b & 0xFF);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(in));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFF)));
}

// Two floats -> one byte of two E2M1 codes (`lo` in bits 0-3), RNE, saturating.
__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
  uint32_t out;
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\t"
      "cvt.u32.u8 %0, b;\n\t}"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out;
}

// Packed bf16 maximum (max.bf16x2); on non-negative non-NaN values it orders
// exactly like the bit patterns.
__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// four bytes (low 8 bits of each argument) -> one word, b0 lowest
__device__ __forceinline__ uint32_t pack4(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  uint32_t lo, hi, r;
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(lo) : "r"(b0), "r"(b1));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(hi) : "r"(b2), "r"(b3));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(r) : "r"(lo), "r"(hi));
  return r;
}

// bf16x2 word times the block's scale (both halves, one mul.rn.ftz.f32x2),
// converted to two E2M1 codes.
__device__ __forceinline__ uint32_t scaled_e2m1x2(uint32_t w, uint64_t os2) {
  uint64_t xv, pv;
  asm("mov.b64 %0, {%1, %2};" : "=l"(xv) : "r"(w << 16), "r"(w & 0xFFFF0000u));
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(pv) : "l"(xv), "l"(os2));
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(pv));
  return f32x2_to_e2m1x2(lo, hi);
}

// g = reciprocal(max(amax, 1e-12)) * 2688 with IEEE rounding at each step,
// as torch evaluates 2688. / t on a device tensor.
__device__ __forceinline__ float encode_scale(float amax) {
  float m = fmaxf(amax, 1e-12f);
  return __fmul_rn(__frcp_rn(m), 2688.0f);
}


// One 16-value block of NVFP4 quantization (the per-block recipe of FlashInfer's
// cvt_warp_fp16_to_fp4, non-TE branch) on its eight bf16x2 words w:
//   vmax = max |x| (exact, bf16);  s8 = e4m3_rn_satfinite(g * (vmax * rcp(6)));
//   os = vmax != 0 ? rcp(float(s8) * rcp(g)) : 0;  code = e2m1_rn_satfinite(x * os)
// with rcp = rcp.approx.ftz.f32 and flush-to-zero products.  r6 = rcp(6), rg = rcp(g)
// are passed in (loop invariants).  Returns s8; c0, c1 get the 16 codes (element 2j in
// the low nibble of byte j).  *sf_value (if given) receives g * (vmax * rcp(6)) before
// the E4M3 conversion and *vmax_bits the block maximum (for saturation checks).
__device__ __forceinline__ uint32_t quantize_block16(const uint32_t (&w)[8], float g, float r6,
                                                     float rg, uint32_t& c0, uint32_t& c1,
                                                     float* sf_value = nullptr,
                                                     uint32_t* vmax_bits = nullptr) {
  const uint32_t m2 = bmax2(bmax2(bmax2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                                  bmax2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu)),
                            bmax2(bmax2(w[4] & 0x7FFF7FFFu, w[5] & 0x7FFF7FFFu),
                                  bmax2(w[6] & 0x7FFF7FFFu, w[7] & 0x7FFF7FFFu)));
  const uint32_t bm = max(m2 & 0xFFFFu, m2 >> 16);   // block max |x|, bf16 bits (exact)
  const float vmax = __uint_as_float(bm << 16);
  const float sfval = mul_ftz(g, mul_ftz(vmax, r6));
  const uint32_t s8 = f32_to_e4m3(sfval);
  const float sfv = e4m3_to_f32(s8);
  // vmax != 0 under flush-to-zero: a subnormal maximum counts as zero
  const float os = (bm >= 0x0080u) ? rcp_approx_ftz(mul_ftz(sfv, rg)) : 0.0f;
  uint64_t os2;
  asm("mov.b64 %0, {%1, %1};" : "=l"(os2) : "f"(os));
  uint32_t byte[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) byte[j] = scaled_e2m1x2(w[j], os2);
  c0 = pack4(byte[0], byte[1], byte[2], byte[3]);
  c1 = pack4(byte[4], byte[5], byte[6], byte[7]);
  if (sf_value != nullptr) *sf_value = sfval;
  if (vmax_bits != nullptr) *vmax_bits = bm;
  return s8;
}

}  // namespace fvq
