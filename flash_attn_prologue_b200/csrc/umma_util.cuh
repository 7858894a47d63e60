// tcgen05 (5th-generation tensor core) and tiled-TMA helpers for sm_100a, as
// inline PTX: single-CTA (cta_group::1) forms, and the CTA-pair
// (cta_group::2) forms a 2-CTA cluster uses to run one M = 256 MMA over the
// shared memory and tensor memory of both SMs. No load uses cluster multicast:
// each CTA loads its own operand halves, and arrivals on the peer's barriers
// use explicit shared::cluster addresses.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tma_util.cuh"

namespace flash_prologue {

// --------------------------------------------------------------------------
// Tensor memory
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
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

// --------------------------------------------------------------------------
// Descriptors
//
// Shared-memory matrix descriptor (64 bit) for a K-major operand tile written by
// TMA with 128-byte swizzling: rows of 128 bytes (64 BF16 along K), 8-row
// swizzle atoms of 1024 bytes. Fields: start address >> 4 (bits 0-13),
// leading-dimension byte offset >> 4 (16-29; unused for swizzled K-major, 1),
// stride-dimension byte offset >> 4 (32-45; 1024 B between 8-row groups),
// descriptor version 1 (bits 46-47), base offset 0 (49-51; tiles are
// 1024-byte aligned), swizzle mode 2 = 128 B (bits 61-63).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// The same for an MN-major operand tile (the backward GEMMs' transposed
// operands): TMA boxes of 64 MN-elements (128 bytes) x 64 K-rows, 128-byte
// swizzle, so a swizzle atom is 8 K-rows x 64 MN-elements (1024 bytes). The
// canonical MN-major layout ((8,n),(8,k)) : ((1,LBO),(8,SBO)) in 16-byte
// units: LBO = bytes between 64-element blocks along MN (one box, `lbo`),
// SBO = bytes between 8-row groups along K (1024). One K = 16 step of an MMA
// advances the start address by two atoms (2048 bytes).
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: BF16 A and B, FP32
// accumulator, both operands K-major, shape M x N (bits: D format 4-5,
// A format 7-9, B format 10-12, A/B major 15/16, N >> 3 at 17-22, M >> 4 at 24-28).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                        // D: FP32
         | (1u << 7)                      // A: BF16
         | (1u << 10)                     // B: BF16
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

// With A and/or B MN-major (bits 15 and 16 of the instruction descriptor).
__host__ __device__ constexpr uint32_t idesc_bf16_f32_major(int M, int N, bool a_mn, bool b_mn) {
  return idesc_bf16_f32(M, N) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive FP32 columns of this thread's TMEM lane (32x32b shape, x32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
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
// 16 consecutive FP32 columns of this thread's TMEM lane (32x32b shape, x16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05.wait::ld that also names the destination registers of the loads it
// completes, so the compiler cannot move a use of them above the wait (loads
// of a later group may be in flight while an earlier group is used).
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&a)[16], uint32_t (&b)[16]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]),
        "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]),
        "+r"(a[14]), "+r"(a[15]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]),
        "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]),
        "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15])
      :
      : "memory");
}

// --------------------------------------------------------------------------
// Tiled TMA load of a 2-D box (no multicast) completing on `bar`.
// c0 is the innermost (contiguous) coordinate; its byte offset must be a
// multiple of 16 (the callers use multiples of 64 BF16 elements).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1),
        "r"(smem_u32(bar))
      : "memory");
}

// Tiled TMA store of a 2-D box from shared memory (bulk-group completion).
// Coordinates are non-negative; c0 is a multiple of 8 BF16 elements (16 bytes).
// Rows outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int32_t c0, int32_t c1,
                                             const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
      ::"l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(src))
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// --------------------------------------------------------------------------
// CTA pairs (2-CTA clusters)

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the variable at `smem_addr` (a shared::cta
// address of this CTA) in the CTA of the cluster with rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// Arrive (release at cluster scope) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Bounded wait (as mbar_wait) with acquire at cluster scope, for barriers that
// the peer CTA arrives on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t i = 0; i < kMaxWaitTries; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(a), "r"(parity), "r"(kSuspendHintNs) : "memory");
    if (done) return true;
  }
  atomicExch(&g_device_error, kDeviceErrorTimeout);
  return false;
}

// Barrier over every thread of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Tensor memory of a CTA pair: issued by one warp (same warp index) in each CTA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D (+)= A * B^T over the pair, issued by one thread of the even CTA: A is
// M = 256 rows, 128 in each CTA's shared memory at the descriptor's offset; B
// is N rows, N/2 in each CTA; each CTA's tensor memory receives its 128 rows.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier at shared::cluster address `bar` (this CTA's
// or the peer's) when every pair MMA this thread issued before has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(bar) : "memory");
}

// Tiled TMA load into this CTA's shared memory whose completion bytes are
// counted on the mbarrier at shared::cluster address `bar`, which may be the
// peer CTA's (no multicast). Same coordinate rules as tma_load_2d.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int32_t c0,
                                                 int32_t c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// 3-D and 4-D forms of tma_load_2d_pair (innermost coordinate first; the
// same alignment rule on c0).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int32_t c0,
                                                 int32_t c1, int32_t c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(bar)
      : "memory");
}
// tma_load_3d_pair with an L2 eviction policy (createpolicy) for the loaded lines.
__device__ __forceinline__ void tma_load_3d_pair_hint(void* dst, const CUtensorMap* map, int32_t c0,
                                                      int32_t c1, int32_t c2, uint32_t bar,
                                                      uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, int32_t c0,
                                                 int32_t c1, int32_t c2, int32_t c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d_pair(void* dst, const CUtensorMap* map, int32_t c0,
                                                 int32_t c1, int32_t c2, int32_t c3, int32_t c4,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3), "r"(c4), "r"(bar)
      : "memory");
}

// 3-D tiled TMA store from shared memory (bulk-group completion; coordinates
// non-negative, rows outside the tensor not written).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int32_t c0, int32_t c1,
                                             int32_t c2, const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];"
      ::"l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
      : "memory");
}

}  // namespace flash_prologue
