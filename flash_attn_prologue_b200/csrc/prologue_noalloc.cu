// Allocation-free backward entry point.
//
// flash_prologue_bwd() needs a caller-provided workspace for the per-CTA
// partial sums of d rmsnorm_weight / d scales. Some callers cannot hand one
// over: runtimes that plan all device memory up front and forbid any
// allocation once they are running, bindings from a host language that can pass
// existing device buffers but has no device allocator of its own, or code that
// runs while another framework's pool holds the device heap. For them,
// flash_prologue_bwd_noalloc() runs the same backward kernels with their
// scratch in a fixed array in this library's device memory (kScratchBytes per
// device, held by every GPU that loads the library until the process exits).
//
// Rules for callers:
//   * The first call on a device looks up the array's device address with that
//     device current (cudaGetSymbolAddress); make that first call before any
//     stream capture.
//   * Every call on a device shares the one array. Calls whose kernels overlap
//     on the GPU (different streams without ordering, or different host threads)
//     race on it; serialise them.
//   * The array keeps the previous call's contents. Nothing needs clearing: the
//     backward writes every partial it later reads.
//   * Problems whose scratch would exceed kScratchBytes are rejected with
//     FLASH_PROLOGUE_ERR_SCRATCH_LIMIT before anything is launched.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <mutex>

#include "../../include/flash_prologue.h"
#include "prologue_host.h"

namespace flash_prologue {
namespace {

constexpr size_t kScratchBytes = size_t(1) << 20;  // 1 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_bwd_scratch[kScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_bwd_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return FLASH_PROLOGUE_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bwd_scratch) != cudaSuccess || !p) return FLASH_PROLOGUE_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FLASH_PROLOGUE_OK;
}

}  // namespace
}  // namespace flash_prologue

extern "C" {

FLASH_PROLOGUE_API int flash_prologue_bwd_noalloc(
    const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
    const float* rmsnorm_weight, const float* scales, const float* sin,
    const int64_t sin_strides[3], const float* cos, const int64_t cos_strides[3],
    const void* grad_q_out, const int64_t gq_strides[4], const void* grad_k_out,
    const int64_t gk_strides[4], void* grad_q, const int64_t dq_strides[4], void* grad_k,
    const int64_t dk_strides[4], float* grad_rmsnorm_weight, float* grad_scales, int64_t B,
    int64_t H, int64_t N, int64_t D, float eps, int dtype, void* stream) {
  size_t need = 0;
  int st = flash_prologue_bwd_workspace_size(B, H, N, D, dtype, &need);
  if (st != FLASH_PROLOGUE_OK) return st;
  if (need > flash_prologue::kScratchBytes) return FLASH_PROLOGUE_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  st = flash_prologue::scratch_address(&scratch);
  if (st != FLASH_PROLOGUE_OK) return st;
  return flash_prologue_bwd(q, q_strides, k, k_strides, rmsnorm_weight, scales, sin, sin_strides,
                            cos, cos_strides, grad_q_out, gq_strides, grad_k_out, gk_strides,
                            grad_q, dq_strides, grad_k, dk_strides, grad_rmsnorm_weight,
                            grad_scales, scratch, flash_prologue::kScratchBytes, B, H, N, D, eps,
                            dtype, stream);
}

}  // extern "C"
