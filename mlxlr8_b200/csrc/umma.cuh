// tcgen05 (5th-generation tensor core) helpers for sm_100a: shared-memory
// matrix descriptors, instruction descriptors, TMEM allocation and loads,
// scale-factor copies, block-scaled MMA, and tiled TMA loads.
//
// Encodings (checked on B200 against a numpy product before use):
//   * smem descriptor: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46),
//     version 1 [46,48), layout type [61,64) (2 = 128-byte swizzle,
//     0 = none).  K-major SW128 tiles are 128-byte rows, 8-row atoms 1 KB
//     apart; the K step inside a row is a plain +32 B on the start field.
//   * block-scaled instruction descriptor (kind::mxf8f6f4): B scale id
//     [4,6), A format [7,10), B format [10,13) (0 = E4M3, 5 = E2M1),
//     N>>3 [17,23), scale type [23] (1 = UE8M0), M>>4 [24,29), A scale id
//     [29,31).  The scale id selects the byte of the 32-bit TMEM cell.
//   * scale factors: 128 rows x 4 K-blocks per 512-byte block, byte
//     (r % 32) * 16 + (r / 32) * 4 + kb; one tcgen05.cp 32x128b.warpx4 puts
//     a block in 4 TMEM columns (lane r % 32 of every sub-partition).
//   * E2M1 operands sit in shared memory as 8 packed bytes (16 values, low
//     nibble first) followed by an 8-byte gap per 16-byte chunk; the TMA
//     type 16U4_ALIGN16B writes that image and counts the packed bytes.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "tma.cuh"

namespace exlr8 {

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// 32 rows of 16 bytes, contiguous (source of a scale-factor copy).
__device__ __forceinline__ uint64_t umma_desc_rows16(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(128 >> 4) << 32) | (static_cast<uint64_t>(1) << 46);
}

constexpr uint32_t kFmtE4M3 = 0, kFmtE2M1 = 5;

// kind::mxf8f6f4 block-scaled descriptor for M = 128, without scale ids.
__host__ __device__ __forceinline__ uint32_t mx_idesc(uint32_t fmt_a, uint32_t fmt_b, int n) {
  return (fmt_a << 7) | (fmt_b << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24);
}

// kind::f16 descriptor, M = 128, bf16 A and B, float32 accumulator.
__host__ __device__ __forceinline__ uint32_t bf16_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_copy_scales(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tc_mma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                          uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %6, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; the caller waits with tc_wait_ld.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// 32 lanes x 8 consecutive 32-bit columns; the caller waits with tc_wait_ld.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 2-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Two-SM (cta_group::2) forms for a cluster of two CTAs on one SM pair.  The
// even CTA (rank 0) issues the MMAs; A comes from both CTAs' shared memory
// (rows 0-127 from rank 0, 128-255 from rank 1), B's N columns are split in
// halves between them, and each CTA's TMEM holds its 128 rows of D.  All
// tcgen05 instructions of such a kernel use cta_group::2.  No multicast.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the variable at local shared address `saddr`
// in the cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}

// All threads of both CTAs.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc2(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_free2(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

// Arrive on the mbarrier at shared::cluster address `bar` (either CTA of
// the pair) once the pair's tcgen05 operations issued so far complete.
__device__ __forceinline__ void tc2_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Each CTA's scale block at `sdesc` (same offset in both) into its own TMEM.
__device__ __forceinline__ void tc2_copy_scales(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tc2_mma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                           uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %6, 0;\n"
      " tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}

// kind::mxf8f6f4 descriptor for the pair's M = 256.
__host__ __device__ __forceinline__ uint32_t mx_idesc_pair(uint32_t fmt_a, uint32_t fmt_b, int n) {
  return (fmt_a << 7) | (fmt_b << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) | ((256u >> 4) << 24);
}

// Tiled TMA load into this CTA's shared memory whose completion is counted
// on the mbarrier at shared::cluster address `bar`, which may be the peer
// CTA's (the pair's MMA issuer waits there for both halves).  No multicast.
__device__ __forceinline__ void tma2_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Remote (or local) arrive on a shared::cluster mbarrier address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait that acquires at cluster scope (arrivals from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t ready;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ready)
        : "r"(smem_u32(bar)), "r"(parity), "n"(100000)
        : "memory");
    if (ready) return true;
  }
  return false;
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

}  // namespace exlr8
