// Host-side structures shared by the C-ABI layer and the kernel launchers.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "prologue_common.cuh"

namespace flash_prologue {

// Index 0 = Q, 1 = K in every two-element array below.
struct FwdArgs {
  const void* x[2];   // inputs
  void* y[2];         // outputs
  RowStrides sx[2], sy[2];
  const float* w;       // [2, D]
  const float* scales;  // [H]
  const float* sin;
  const float* cos;
  TableStrides ssin, scos;
  int64_t B, N;
  int H;
  float eps;
  Geometry g;
};

struct BwdArgs {
  const void* x[2];   // q, k
  const void* gy[2];  // upstream gradients of q_out, k_out
  void* dx[2];        // dq, dk
  RowStrides sx[2], sgy[2], sdx[2];
  const float* w;
  const float* scales;
  const float* sin;
  const float* cos;
  TableStrides ssin, scos;
  float* partials;  // [grid, 2*D + H] per-CTA partial sums
  int64_t B, N;
  int H;
  float eps;
  Geometry g;
};

// Geometry of a problem (layout-dependent, device-independent).
Geometry plan_geometry(int64_t B, int64_t H, int64_t N, int D, bool heads_inner);

// Persistent grid for a kernel: min(items, SMs x resident CTAs per SM).
int64_t persistent_grid(const void* kernel, size_t smem_bytes, int64_t n_items);

// Launchers; return a cudaError_t from the launch.
cudaError_t launch_fwd(const FwdArgs& a, int dtype, int D, bool vec, cudaStream_t stream);

// Grid the backward kernel uses for this geometry on the current device.
int64_t bwd_grid(const Geometry& g, int H, int D, int dtype, bool vec);
size_t bwd_smem_bytes(int H, int D);
cudaError_t launch_bwd(const BwdArgs& a, float* dw, float* ds, int dtype, int D, bool vec,
                       cudaStream_t stream);

}  // namespace flash_prologue
