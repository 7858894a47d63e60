// TMA (bulk and tensor copies) and mbarrier helpers for sm_100a, written as inline PTX.
//
// Every wait is bounded: after kMaxWaitTries suspended polls (a few seconds in
// total) the waiter records kDeviceErrorTimeout in the library's device error
// word and gives up, so a protocol bug ends the kernel instead of hanging the
// GPU. flash_prologue_device_error() reads (and optionally clears) the word.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace flash_prologue {

constexpr int kDeviceErrorTimeout = 1;
constexpr uint32_t kMaxWaitTries = 1u << 22;  // x suspend hint below: about 4 s
constexpr uint32_t kSuspendHintNs = 1000;

// Device error word of the waits in this translation unit (0 = no error). The
// library is built without relocatable device code, so every .cu file that
// includes this header has its own word and its own host-side reader.
static __device__ int g_device_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Waits for the phase with the given parity to complete. Returns false (and
// records a device error) if it did not within the bound.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t i = 0; i < kMaxWaitTries; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(a), "r"(parity), "r"(kSuspendHintNs) : "memory");
    if (done) return true;
  }
  atomicExch(&g_device_error, kDeviceErrorTimeout);
  return false;
}

// L2 eviction policies for bulk copies. The streamed prologue tiles use the
// normal policy: evict_first on them measured 1% (backward) to 4% (forward)
// slower at C2 sizes.
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Global -> shared bulk copy (no multicast) completing on `bar` with a byte
// count. Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled TMA load of a 5-D box (no multicast) completing on `bar`, with an L2
// cache policy. c0 is the innermost coordinate: its byte offset must be a
// multiple of 16 (the prologue kernels always pass 0). The shared-memory
// destination is 128-byte aligned.
__device__ __forceinline__ void tma_load_5d_hint(void* dst, const CUtensorMap* map, int32_t c0,
                                                 int32_t c1, int32_t c2, int32_t c3, int32_t c4,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3), "r"(c4), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled TMA store of a 5-D box from shared memory (bulk-group completion), the
// inverse of tma_load_5d_hint: c0 is 0 or a 16-byte multiple, no coordinate is
// negative, and rows outside the tensor are not written.
__device__ __forceinline__ void tma_store_5d(const CUtensorMap* map, const void* src, int32_t c0,
                                             int32_t c1, int32_t c2, int32_t c3, int32_t c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4, %5}], [%6];"
      ::"l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
        "r"(smem_u32(src))
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until the committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until at most N of the most recently committed bulk-store groups are
// still reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until the committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Makes this thread's generic-proxy shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Warpgroup register reallocation: all 128 threads of a warpgroup execute the
// same instruction. An increase waits until the block's pool (registers per
// thread at launch x threads) has room, so the split must fit that pool.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Barrier over the consumer warps only (the producer warp does not take part).
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

}  // namespace flash_prologue
