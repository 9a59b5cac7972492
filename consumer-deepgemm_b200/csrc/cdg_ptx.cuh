// Thin inline-PTX wrappers for the sm_100a features the grouped GEMM uses:
// mbarriers, TMA (tiled tensor loads and 1-D bulk copies), TMEM allocation,
// tcgen05 block-scaled MMA, tcgen05.cp / tcgen05.ld and the tcgen05 fences.
//
// Every wait in this file is bounded: a wait that has not completed after
// CDG_WAIT_TIMEOUT_NS of wall time (read from %globaltimer) records
// CDG_STATUS_TIMEOUT in the caller's status word and returns false, so a broken
// pipeline ends the kernel with an error code instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#ifndef CDG_WAIT_TIMEOUT_NS
#define CDG_WAIT_TIMEOUT_NS 2000000000ull  // 2 s
#endif

namespace cdg {

// Status bits written by device code (OR-ed into a caller-visible word).
enum : int {
  kStatusTimeout = 1,       // an mbarrier wait exceeded CDG_WAIT_TIMEOUT_NS
  kStatusBadIndex = 2,      // an index a kernel computed fell outside its buffer
};

// Sticky per-device record of device-side errors, kept by the library itself: every bounded
// wait that gives up ORs its status bit into [0] and leaves the first wait code in [1],
// whichever workspace the call used (caller memory, or the no-allocation entry's static
// scratch).  cdg_device_status() reads and optionally clears it.  One copy per translation
// unit that includes this header (the host side of that unit reads its own copy).
static __device__ int g_sticky_status[2];

__device__ __forceinline__ void record_timeout(int* status, int where) {
  if (status) {
    atomicOr(status, kStatusTimeout);
    atomicCAS(status + 1, 0, where);
  }
  atomicOr(&g_sticky_status[0], kStatusTimeout);
  atomicCAS(&g_sticky_status[1], 0, where);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity), "r"(0x989680u)  // suspend-time hint (ns)
      : "memory");
  return done != 0;
}

// Non-blocking test of the phase with the given parity (acquire at CTA scope).  The bounded
// waits below probe with it first: on a phase that has already completed it returns sooner
// than try_wait (in the prefill kernels' issuing warp, ~125 against ~185 cycles per wait).
__device__ __forceinline__ bool mbar_test(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (and sets
// kStatusTimeout) when the wait gives up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_test(addr, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (global_timer_ns() - t0 > CDG_WAIT_TIMEOUT_NS) {
      if (status) atomicOr(status, kStatusTimeout);
      atomicOr(&g_sticky_status[0], kStatusTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y,
                                            int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Warm L2 with one box of a tiled tensor (no shared memory involved).
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(tmap)),
               "r"(x), "r"(y)
               : "memory");
}

// Warm L2 with `bytes` (multiple of 16) starting at a 16-byte aligned global address.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}

// Plain 1-D bulk copy global -> shared (size and both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels launched with programmatic stream serialization may be scheduled before the
// previous kernel of the stream finished; they wait here before reading its results.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the stream be scheduled (it still waits for this grid's end).
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- CTA pairs (clusters of 2)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of this CTA's shared variable `p` in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

// Arrive (release at cluster scope) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity), "r"(0x989680u)
      : "memory");
  return done != 0;
}

// Non-blocking test of the phase with the given parity (acquire at cluster scope).
__device__ __forceinline__ bool mbar_test_cluster(uint64_t* bar, uint32_t parity) {
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

// Bounded wait whose completion may come from the other CTA of the pair (acquire at
// cluster scope).  Returns false (and sets kStatusTimeout) when it gives up; the first
// wait to give up also leaves `where` (a caller-chosen code naming the wait) in status[1].
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status, int where = 0) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_test_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_cluster(addr, parity)) return true;
    if (global_timer_ns() - t0 > CDG_WAIT_TIMEOUT_NS) {
      record_timeout(status, where);
      return false;
    }
  }
}

// Code naming a wait for mbar_wait_cluster: role (1 producer/empty, 2 issuer/tempty,
// 3 issuer/full (or sfready), 4 epilogue/tfull, 5 issuer/done, 6 scale copier/full (or the
// TMEM scale slot), 7 scale-atom producer/slot free; 15 is not a wait: the TMEM allocation
// did not start at column 0), CTA rank or issuer, stage, phase, step.
__device__ __forceinline__ int wait_code(int role, int who, int stage, uint32_t phase, int step) {
  const uint32_t c = (static_cast<uint32_t>(role & 15) << 28) | (static_cast<uint32_t>(who & 15) << 24) |
                     (static_cast<uint32_t>(stage & 255) << 16) | ((phase & 1u) << 15) |
                     static_cast<uint32_t>(step & 0x7fff);
  return static_cast<int>(c);  // the bit pattern; roles >= 8 read as negative int32
}

// Tiled TMA loads into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (`cluster_bar`, a shared::cluster address).  No
// multicast: each CTA loads its own tiles.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint32_t cluster_bar, int32_t x,
                                                 int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const void* tmap, uint32_t cluster_bar, int32_t x,
                                                 int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(cluster_bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(void* dst, const void* tmap, uint32_t cluster_bar, int32_t x,
                                                 int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(cluster_bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads
// (TMA, tcgen05.cp, tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive on `bar` once every previously issued tcgen05 async op of this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Copy one 128-row x 4-byte scale-factor atom (512 B, the 32x128b pattern)
// from shared memory into 4 TMEM columns, replicated to the 4 lane quadrants.
__device__ __forceinline__ void tc_cp_sf_atom(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem] with per-32-K UE8M0 scale factors in TMEM.
__device__ __forceinline__ void tc_mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// ---- CTA-pair forms (cta_group::2): issued by the even CTA of the pair, acting on both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// Arrive on the mbarrier at the same offset in each CTA of `cta_mask` once every
// previously issued tcgen05 async op of this thread completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(smem_u32(bar)), "h"(cta_mask)
      : "memory");
}

// Scale-factor atom copy for both CTAs: each CTA's atom at this shared-memory offset
// goes to the same TMEM columns of that CTA.
__device__ __forceinline__ void tc_cp_sf_atom_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// D (+)= A * B over the pair: M = 256 (rows 0-127 from the even CTA's A tile, 128-255
// from the odd CTA's), B's N rows split in halves between the CTAs, D's rows in the
// TMEM of the CTA that holds them.
__device__ __forceinline__ void tc_mma_mxf8f6f4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                     uint32_t accumulate, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// ---- warp-wide forms: every lane of the warp executes the call with the same
// (warp-uniform) operands and the instruction is issued by the lane elect.sync picks (the
// same lane every time, so its commits track its own tcgen05 operations).  A loop run by
// the whole warp this way issues tcgen05.mma at about 50 cycles each; the same loop in a
// branch taken by one lane needed about 75.
__device__ __forceinline__ void tc_mma_mxf8f6f4_pair_warp(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                          uint32_t idesc, uint32_t accumulate, uint32_t sfa_tmem,
                                                          uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

__device__ __forceinline__ void tc_commit_pair_warp(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}"
      ::"r"(smem_u32(bar)), "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ void tc_cp_sf_atom_pair_warp(uint32_t taddr, uint64_t sdesc) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;\n\t}"
      ::"r"(taddr), "l"(sdesc)
      : "memory");
}

// Bounded wait for a barrier of this CTA, default (CTA) scope: for barriers completed by
// TMA transactions or tcgen05.commit, which order the data the following tcgen05 operations
// read.  Cheaper than the cluster-scope acquire of mbar_wait_cluster.
__device__ __forceinline__ bool mbar_wait_cta(uint64_t* bar, uint32_t parity, int* status, int where = 0) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_test(addr, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (global_timer_ns() - t0 > CDG_WAIT_TIMEOUT_NS) {
      record_timeout(status, where);
      return false;
    }
  }
}

// mbar_wait_cta by every lane of the warp; true for all lanes only if no lane gave up.
__device__ __forceinline__ bool mbar_wait_cta_warp(uint64_t* bar, uint32_t parity, int* status, int where = 0) {
  const bool ok = mbar_wait_cta(bar, parity, status, where);
  return __all_sync(0xffffffffu, ok);
}

// mbar_wait_cluster by every lane of the warp; true for all lanes only if no lane gave up.
__device__ __forceinline__ bool mbar_wait_cluster_warp(uint64_t* bar, uint32_t parity, int* status, int where = 0) {
  const bool ok = mbar_wait_cluster(bar, parity, status, where);
  return __all_sync(0xffffffffu, ok);
}

// Load 16 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 lanes x 16 columns from TMEM lane `taddr.lane`, column `taddr.col` (shape 16x256b, x2).
// Thread t receives, for lane l = t/4 and column c = 2*(t%4):
//   r0, r1 = (l, c), (l, c+1);  r2, r3 = (l+8, c), (l+8, c+1);  r4..r7 = the same at c+8.
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// Four 8x8 b16 matrices, stored transposed: register k of thread t holds row t/4, columns
// 2*(t%4) and +1 (low half first) of matrix k; row i of the stored transpose of matrix k
// (16 bytes) goes to the address given by thread 8*k + i.
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, uint32_t m0, uint32_t m1, uint32_t m2, uint32_t m3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(m0), "r"(m1),
               "r"(m2), "r"(m3)
               : "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (tcgen05 format, version 1): K-major operand
// tile whose rows are 128 bytes, stored with the 128-byte swizzle; 8-row core
// groups are 1024 bytes apart.  `addr` must lie in a 1024-byte aligned tile
// (plus a k offset of a multiple of 32 bytes within the swizzle row).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);          // start address
  d |= static_cast<uint64_t>(0) << 16;                         // leading byte offset (unused for SW128 K-major)
  d |= static_cast<uint64_t>((1024u >> 4) & 0x3FFFu) << 32;    // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;                         // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                         // layout: 128-byte swizzle
  return d;
}

// Descriptor of a scale-factor atom for tcgen05.cp: no swizzle, 8 rows x 16 B
// core groups 128 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sf(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((128u >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::mxf8f6f4 block_scale, FP32 accumulate,
// both operands K-major, UE8M0 scales.
//   a_fmt/b_fmt: 0 = E4M3, 1 = E5M2, 3 = E2M3, 4 = E3M2, 5 = E2M1
__device__ __forceinline__ uint32_t idesc_mxf8f6f4(uint32_t a_fmt, uint32_t b_fmt, uint32_t m, uint32_t n,
                                                   uint32_t a_sf_id, uint32_t b_sf_id) {
  uint32_t d = 0;
  d |= (b_sf_id & 3u) << 4;
  d |= (a_fmt & 7u) << 7;
  d |= (b_fmt & 7u) << 10;
  // bits 13,14 negate = 0; bits 15,16 major = 0 (K-major)
  d |= ((n >> 3) & 0x3Fu) << 17;
  d |= 1u << 23;  // scale format UE8M0
  d |= ((m >> 4) & 0x1Fu) << 24;
  d |= (a_sf_id & 3u) << 29;
  return d;
}

}  // namespace cdg
