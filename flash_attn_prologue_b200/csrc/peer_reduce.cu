// Data-parallel finalize of the backward's parameter gradients over peer memory.
//
// The backward kernel leaves one [2*D + H] FP32 partial per CTA; a finalize
// kernel adds them in a fixed order into d rmsnorm_weight and d scales. With
// data-parallel training that [C] vector must then be summed over the ranks.
// peer_finalize_kernel does both in one launch, over NVLink / NVSwitch peer
// memory instead of a library collective:
//
//   1. block b adds the CTA partials of columns 32b .. 32b + 31 in the order of
//      the single-GPU finalize (warp w takes rows w, w + 8, ..., then the eight
//      warp sums in warp order), so a one-rank group gives its bits exactly;
//   2. its 32 sums go to row `rank` of every rank's exchange buffer (plain
//      stores to the peers' mapped memory), then a system-scope fence;
//   3. one thread releases the block's flag (the call's epoch) in every rank's
//      flag array, then waits -- bounded -- until every rank's flag for this
//      block has arrived in its own array;
//   4. the block adds the world rows of its own buffer in rank order.
//
// Every rank therefore sums the same values in the same order: identical bits
// on every rank and run to run. Calls alternate between two halves of the
// buffers (epoch parity): a rank writes half p of call e + 2 only after every
// rank's flag of call e + 1 reached it, which each rank sets after finishing
// its reads of call e. A wait that runs out records the device error word and
// writes NaN, so a missing rank cannot return a plausible partial sum. Each
// wait is bounded by time (the descriptor's wait_ms, read from %globaltimer)
// and by a poll count. No TMA and no multicast: plain loads and stores.
#include <cstring>
#include <mutex>

#include "../../include/flash_prologue.h"
#include "prologue_host.h"

namespace flash_prologue {
namespace {

constexpr int kPeerThreads = 256;
constexpr int kPeerWarps = kPeerThreads / 32;
constexpr uint32_t kPeerWaitPolls = 1u << 26;  // backstop to the time bound
constexpr int kPeerDefaultWaitMs = 2000;
static __device__ int g_peer_error = 0;

struct PeerArgs {
  const float* partials[FLASH_PROLOGUE_MAX_PEERS];  // by emulated rank slot (blockIdx.y)
  float* dw[FLASH_PROLOGUE_MAX_PEERS];
  float* ds[FLASH_PROLOGUE_MAX_PEERS];
  float* data[FLASH_PROLOGUE_MAX_PEERS];     // every rank's exchange buffer, as mapped here
  uint32_t* flags[FLASH_PROLOGUE_MAX_PEERS];
  int64_t G;
  int C, two_d, world, rank0, max_cols, nblk;
  uint32_t epoch;
  uint64_t wait_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ float ld_relaxed_sys(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kPeerThreads) peer_finalize_kernel(const __grid_constant__ PeerArgs a) {
  __shared__ float part[kPeerWarps][32];
  __shared__ int arrived;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int slot = blockIdx.y;  // 0, or the emulated rank
  const int rank = a.rank0 + slot;
  const int blk = blockIdx.x;
  const int col = blk * 32 + lane;
  const uint32_t half = a.epoch & 1u;

  // 1. this rank's fixed-order sum of its CTA partials
  const float v = col < a.C ? strided_column_sum(a.partials[slot], a.G, a.C, col, warp, kPeerWarps) : 0.f;
  part[warp][lane] = v;
  __syncthreads();
  if (warp == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kPeerWarps; ++w) s = __fadd_rn(s, part[w][lane]);
    // 2. into row `rank` of every rank's buffer
    if (col < a.C)
      for (int p = 0; p < a.world; ++p)
        a.data[p][((size_t)half * a.world + rank) * a.max_cols + col] = s;
    __threadfence_system();
  }
  __syncthreads();
  // 3. release this block's flag everywhere, wait for everyone's here
  if (threadIdx.x == 0) {
    for (int p = 0; p < a.world; ++p)
      st_release_sys(a.flags[p] + ((size_t)half * a.world + rank) * a.nblk + blk, a.epoch);
    const uint32_t* mine = a.flags[rank] + (size_t)half * a.world * a.nblk;
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    uint32_t polls = 0;
    for (int j = 0; j < a.world && ok; ++j) {
      while (ld_acquire_sys(mine + (size_t)j * a.nblk + blk) != a.epoch) {
        if (++polls >= kPeerWaitPolls || globaltimer_ns() - t0 > a.wait_ns) {
          ok = 0;
          break;
        }
        __nanosleep(128);
      }
    }
    if (!ok) atomicExch(&g_peer_error, 1);
    arrived = ok;
  }
  __syncthreads();
  // 4. the world rows in rank order
  if (warp == 0 && col < a.C) {
    const float* mine = a.data[rank] + (size_t)half * a.world * a.max_cols;
    float s = ld_relaxed_sys(mine + col);  // rank 0's row, so one rank returns its own bits (-0 included)
    for (int j = 1; j < a.world; ++j) s = __fadd_rn(s, ld_relaxed_sys(mine + (size_t)j * a.max_cols + col));
    if (!arrived) s = __int_as_float(0x7fc00000);
    if (col < a.two_d) a.dw[slot][col] = s;
    else a.ds[slot][col - a.two_d] = s;
  }
}

bool peers_ok(const flash_prologue_peers* p, int C) {
  if (!p || p->world < 1 || p->world > FLASH_PROLOGUE_MAX_PEERS || p->rank < 0 || p->rank >= p->world)
    return false;
  if (p->max_cols < C || p->max_cols % 32 != 0 || p->wait_ms < 0 || p->wait_ms > 60000) return false;
  for (int r = 0; r < p->world; ++r)
    if (!p->data[r] || !p->flags[r]) return false;
  return true;
}

PeerArgs peer_args(const flash_prologue_peers* p, int64_t G, int C, int two_d, uint32_t epoch) {
  PeerArgs a{};
  a.G = G;
  a.C = C;
  a.two_d = two_d;
  a.world = p->world;
  a.max_cols = p->max_cols;
  a.nblk = p->max_cols / 32;
  a.epoch = epoch;
  a.wait_ns = (uint64_t)(p->wait_ms ? p->wait_ms : kPeerDefaultWaitMs) * 1000000ull;
  for (int r = 0; r < p->world; ++r) {
    a.data[r] = p->data[r];
    a.flags[r] = p->flags[r];
  }
  return a;
}

// cuMemGetAddressRange through the runtime's driver entry-point query (the
// library does not link libcuda).
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

}  // namespace

cudaError_t launch_bwd_reduce(const float* partials, int64_t G, int C, int two_d, float* dw, float* ds,
                              const BwdReduce& red, cudaStream_t stream) {
  if (!red.peers) return launch_bwd_finalize(partials, G, C, two_d, dw, ds, stream);
  if (!peers_ok(red.peers, C) || red.epoch == 0) return cudaErrorInvalidValue;
  PeerArgs a = peer_args(red.peers, G, C, two_d, red.epoch);
  a.rank0 = red.peers->rank;
  a.partials[0] = partials;
  a.dw[0] = dw;
  a.ds[0] = ds;
  return launch_kernel(peer_finalize_kernel, dim3((unsigned)a.nblk, 1), dim3(kPeerThreads), 0, stream, a);
}

cudaError_t read_peer_device_error(int* value, bool reset) {
  cudaError_t err = cudaMemcpyFromSymbol(value, g_peer_error, sizeof(int));
  if (err != cudaSuccess || !reset) return err;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_peer_error, &zero, sizeof(int));
}

}  // namespace flash_prologue

using namespace flash_prologue;

extern "C" {

FLASH_PROLOGUE_API int flash_prologue_peer_buffer_bytes(int32_t world, int32_t max_cols, size_t* data_bytes,
                                                        size_t* flag_bytes) {
  if (!data_bytes || !flag_bytes || world < 1 || world > FLASH_PROLOGUE_MAX_PEERS || max_cols < 32 ||
      max_cols % 32 != 0)
    return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  *data_bytes = (size_t)2 * world * max_cols * sizeof(float);
  *flag_bytes = (size_t)2 * world * (max_cols / 32) * sizeof(uint32_t);
  return FLASH_PROLOGUE_OK;
}

FLASH_PROLOGUE_API int flash_prologue_ipc_handle(const void* dev_ptr, void* handle, int64_t* offset) {
  if (!dev_ptr || !handle || !offset) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  AddressRangeFn range = address_range_fn();
  if (!range) return FLASH_PROLOGUE_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return FLASH_PROLOGUE_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return FLASH_PROLOGUE_ERR_CUDA;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return FLASH_PROLOGUE_OK;
}

FLASH_PROLOGUE_API int flash_prologue_ipc_open(const void* handle, int64_t offset, void** dev_ptr) {
  if (!handle || !dev_ptr || offset < 0) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return FLASH_PROLOGUE_ERR_CUDA;
  *dev_ptr = static_cast<char*>(base) + offset;
  return FLASH_PROLOGUE_OK;
}

FLASH_PROLOGUE_API int flash_prologue_ipc_close(void* dev_ptr, int64_t offset) {
  if (!dev_ptr || offset < 0) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(static_cast<char*>(dev_ptr) - offset) == cudaSuccess ? FLASH_PROLOGUE_OK
                                                                                    : FLASH_PROLOGUE_ERR_CUDA;
}

FLASH_PROLOGUE_API int flash_prologue_peer_reduce_emulated(const float* const* partials, int64_t G, int32_t C,
                                                           int32_t two_d, float* const* dw, float* const* ds,
                                                           const flash_prologue_peers* peers, uint32_t epoch,
                                                           void* stream) {
  if (!partials || !dw || !ds || G < 1 || C < 1 || two_d < 0 || two_d > C || epoch == 0 || !peers_ok(peers, C))
    return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  PeerArgs a = peer_args(peers, G, C, two_d, epoch);
  a.rank0 = 0;
  for (int r = 0; r < peers->world; ++r) {
    if (!partials[r] || !dw[r] || !ds[r]) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
    a.partials[r] = partials[r];
    a.dw[r] = dw[r];
    a.ds[r] = ds[r];
  }
  // The emulated ranks' blocks wait on one another: a cooperative launch
  // guarantees they are all resident at once (or fails instead of starting).
  void* args[] = {&a};
  const cudaError_t err =
      cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&peer_finalize_kernel),
                                  dim3((unsigned)a.nblk, (unsigned)peers->world), dim3(kPeerThreads), args, 0,
                                  static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
}

}  // extern "C"
