// Strided row copy: dst[i0, i1, i2, :] = src[i0, i1, i2, :] for rows of
// `row_bytes` contiguous bytes (a multiple of 16) under three outer
// dimensions with arbitrary byte strides. It moves the V slot of a fused QKV
// tensor (or of its gradient) to or from a separate tensor -- the copies next
// to the prologue kernels, which a generic elementwise copy runs at a third of
// the copy bandwidth on these layouts.
//
// Each warp copies whole rows: its lanes split into groups of G lanes per row
// (G = min(32, row_bytes / 16)), every lane moves 16-byte chunks, up to four
// in flight, with read-only loads and streaming stores. The grid is a small
// multiple of the SM count and walks the rows with a grid stride.
#include "../../include/flash_prologue.h"
#include "prologue_host.h"

namespace flash_prologue {
namespace {

struct CopyArgs {
  const char* src;
  char* dst;
  int64_t dims[3];      // outer extents (i0, i1, i2), i2 fastest
  int64_t ss[3], ds[3];  // byte strides of src and dst
  int64_t rows;         // dims[0] * dims[1] * dims[2]
  int64_t chunks;       // 16-byte chunks per row
  int lanes_per_row;    // G, a power of two
};

__global__ void __launch_bounds__(256) copy_rows_kernel(const CopyArgs a) {
  const int lane = threadIdx.x & 31;
  const int G = a.lanes_per_row;
  const int sub = lane / G;          // which row of the warp's group
  const int gl = lane % G;           // lane within the row
  const int rows_per_warp = 32 / G;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp0 * rows_per_warp + sub; r < a.rows; r += nwarps * rows_per_warp) {
    const int64_t i2 = r % a.dims[2];
    const int64_t t = r / a.dims[2];
    const int64_t i1 = t % a.dims[1];
    const int64_t i0 = t / a.dims[1];
    const uint4* s = reinterpret_cast<const uint4*>(a.src + i0 * a.ss[0] + i1 * a.ss[1] + i2 * a.ss[2]);
    uint4* d = reinterpret_cast<uint4*>(a.dst + i0 * a.ds[0] + i1 * a.ds[1] + i2 * a.ds[2]);
    int64_t c = gl;
    for (; c + 3 * G < a.chunks; c += 4 * G) {
      const uint4 v0 = __ldg(s + c), v1 = __ldg(s + c + G), v2 = __ldg(s + c + 2 * G),
                  v3 = __ldg(s + c + 3 * G);
      __stcs(d + c, v0);
      __stcs(d + c + G, v1);
      __stcs(d + c + 2 * G, v2);
      __stcs(d + c + 3 * G, v3);
    }
    for (; c < a.chunks; c += G) __stcs(d + c, __ldg(s + c));
  }
}

// [first, last] bytes a view touches: base plus each outer dimension's extent
// times the magnitude of its stride (negative strides reach below the base).
void byte_span(const void* base, const int64_t strides[3], const int64_t dims[3], int64_t row_bytes,
               uintptr_t* lo, uintptr_t* hi) {
  int64_t below = 0, above = row_bytes - 1;
  for (int i = 0; i < 3; ++i) {
    const int64_t reach = (dims[i] - 1) * strides[i];
    if (reach < 0) below += reach; else above += reach;
  }
  *lo = reinterpret_cast<uintptr_t>(base) + below;
  *hi = reinterpret_cast<uintptr_t>(base) + above;
}

bool byte_span_overlap(const void* src, const int64_t ss[3], const void* dst, const int64_t ds[3],
                       const int64_t dims[3], int64_t row_bytes) {
  uintptr_t slo, shi, dlo, dhi;
  byte_span(src, ss, dims, row_bytes, &slo, &shi);
  byte_span(dst, ds, dims, row_bytes, &dlo, &dhi);
  return slo <= dhi && dlo <= shi;
}

}  // namespace
}  // namespace flash_prologue

using namespace flash_prologue;

extern "C" {

FLASH_PROLOGUE_API int flash_prologue_copy_rows(const void* src, const int64_t src_strides[3],
                                                void* dst, const int64_t dst_strides[3],
                                                const int64_t dims[3], int64_t row_bytes,
                                                void* stream) {
  if (!src_strides || !dst_strides || !dims) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (dims[0] < 0 || dims[1] < 0 || dims[2] < 0 || row_bytes < 0)
    return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  const int64_t rows = dims[0] * dims[1] * dims[2];
  if (rows == 0 || row_bytes == 0) return FLASH_PROLOGUE_OK;
  if (!src || !dst) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (row_bytes % 16 != 0) return FLASH_PROLOGUE_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u)
    return FLASH_PROLOGUE_ERR_ALIGNMENT;
  for (int i = 0; i < 3; ++i)
    if ((dims[i] > 1 && ((src_strides[i] | dst_strides[i]) & 15) != 0))
      return FLASH_PROLOGUE_ERR_ALIGNMENT;
  // src is read through the read-only (non-coherent) path while dst is written,
  // so the two must not overlap: byte ranges that do are rejected.
  if (byte_span_overlap(src, src_strides, dst, dst_strides, dims, row_bytes))
    return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  CopyArgs a{};
  a.src = static_cast<const char*>(src);
  a.dst = static_cast<char*>(dst);
  for (int i = 0; i < 3; ++i) {
    a.dims[i] = dims[i];
    a.ss[i] = src_strides[i];
    a.ds[i] = dst_strides[i];
  }
  a.rows = rows;
  a.chunks = row_bytes / 16;
  int G = 1;
  while (G < 32 && G < a.chunks) G *= 2;
  a.lanes_per_row = G;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return FLASH_PROLOGUE_ERR_CUDA;
  const int64_t rows_per_block = 8 * (32 / G);
  const int64_t want = (rows + rows_per_block - 1) / rows_per_block;
  const int64_t cap = 8LL * sms;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  return launch_kernel(copy_rows_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), a) ==
                 cudaSuccess
             ? FLASH_PROLOGUE_OK
             : FLASH_PROLOGUE_ERR_CUDA;
}

}  // extern "C"
