// Host-side encoding of TMA tensor maps (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry-point query so the library does not link
// libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace flash_prologue {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Looked up once per process (a function-local static: thread-safe initialisation).
inline EncodeTiledFn tensor_map_encoder() {
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return EncodeTiledFn(nullptr);
  }();
  return fn;
}

// Tiled map of a rank-R tensor: dims[0] innermost (contiguous), byte strides
// of dims 1 .. R-1 in strides_bytes[0 .. R-2], a box of box[0..R-1] elements,
// the given swizzle, zero fill out of bounds. False if the driver rejects it
// (alignment, stride or box rules).
inline bool encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank,
                              const void* base, const uint64_t* dims,
                              const uint64_t* strides_bytes, const uint32_t* box,
                              CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = tensor_map_encoder();
  if (!fn || rank < 1 || rank > 5) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  auto encode = [&] {
    return fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  static thread_local bool bound = false;
  if (r != CUDA_SUCCESS && !bound) {
    // The driver call needs a context bound to the calling thread, and a thread
    // whose first CUDA call this is (an autograd worker, say) has none yet: bind
    // the current device's primary context through the runtime (once per
    // thread) and retry, instead of failing and sending the call down the
    // register path, which groups the parameter-gradient sums differently.
    bound = true;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = encode();
  }
  return r == CUDA_SUCCESS;
}

}  // namespace flash_prologue
