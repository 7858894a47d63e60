// Host-side structures shared by the C-ABI layer and the kernel launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <tuple>
#include <type_traits>
#include <utility>

#include "prologue_common.cuh"

struct flash_prologue_peers;  // include/flash_prologue.h

namespace flash_prologue {

// Launches fn<<<grid, block, smem, stream>>>(args...) through cudaLaunchKernel
// and returns the error of this launch only (a launch with <<<>>> reports
// through cudaGetLastError, which would also return -- and clear -- an error
// left pending by unrelated earlier work).
template <typename... P, typename... A>
inline cudaError_t launch_kernel(void (*fn)(P...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t stream, A&&... args) {
  static_assert(sizeof...(P) == sizeof...(A), "kernel argument count");
  std::tuple<std::decay_t<P>...> vals(std::forward<A>(args)...);
  return std::apply(
      [&](auto&... v) {
        void* ptrs[] = {static_cast<void*>(&v)..., nullptr};
        return cudaLaunchKernel(reinterpret_cast<const void*>(fn), grid, block, ptrs, smem, stream);
      },
      vals);
}

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
  float* rms[2];        // optional: r = 1/sqrt(mean(x^2)+eps) per row, FP32 [B, H, N]
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
  // Inverse backward only: x[] are the forward OUTPUTS and rms[] their saved
  // r per row (FP32 [B, H, N]); the normalised rows are rebuilt from them.
  const float* rms[2];
  int64_t B, N;
  int H;
  float eps;
  Geometry g;
};

// ---------------------------------------------------------------------------
// TMA pipelined path.
constexpr int kTmaConsumerWarps = 8;                       // 0-3: Q rows, 4-7: K rows
constexpr int kTmaThreads = (kTmaConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kTmaTileBytes = 8192;                        // per streamed tensor per stage
// Pipeline stages of the forward / backward kernels. Compile-time, so the
// kernels' stage index and barrier phase (k % S, k / S) cost a multiply and a
// shift instead of an integer division per tile.
constexpr int kTmaFwdStages = 3;
constexpr int kTmaBwdStages = 3;

// Bytes of one pipeline stage: `nt` streamed tiles, then the sin and cos rows,
// rounded up so that every stage (each TMA destination) stays 128-byte aligned.
__host__ __device__ constexpr int tma_stage_bytes(int nt, int table_bytes) {
  return (nt * kTmaTileBytes + 2 * table_bytes + 127) & ~127;
}
// The forward that saves r adds, after each stage's tables, the tile's r values
// ([tensor][row], FP32) that the producer writes out once the stage is free.
__host__ __device__ constexpr int tma_r_area_bytes(int rows) { return (2 * rows * 4 + 127) & ~127; }

// The backward kernel runs the 8 consumer warps (warpgroups 0-1) beside a
// whole producer warpgroup (warp 8 issues the copies; warps 9-11 leave once
// the group has given its registers back). It is launched at
// kTmaBwdLaunchRegs registers per thread (two CTAs per SM: 2 x 384 x 80 fit in
// the 65,536-register file); the producer group then drops to 32 and the
// consumers rise to 104, which the block's own allocation covers exactly.
constexpr int kTmaBwdThreads = (kTmaConsumerWarps + 4) * 32;
constexpr int kTmaBwdLaunchRegs = 80;
constexpr int kTmaBwdProducerRegs = 32;
constexpr int kTmaBwdConsumerRegs = 104;
static_assert(4 * 32 * kTmaBwdProducerRegs + kTmaConsumerWarps * 32 * kTmaBwdConsumerRegs <=
                  kTmaBwdThreads * kTmaBwdLaunchRegs,
              "backward register split exceeds the block's launch allocation");

struct TmaPlan {
  int heads_inner;      // inner row dim: 1 = heads, 0 = positions
  int ti, log2_ti;      // rows per tile along the inner dim (power of two)
  int to;               // rows per tile along the outer dim; ti * to = tile rows
  int P;                // sin/cos rows per tile
  int stages;
  int64_t inner_ext, outer_ext;
  int64_t n_ib, n_ob, n_tiles;  // tiles = B * n_ob * n_ib, inner block fastest
  Radix4 radix;                  // digits (inner block, outer block, b); set at launch
};

// One streamed input, read by tiled TMA loads. The tensor map views it as 5-D
// {D/2, inner, outer, 2, B}: a half row, the inner and outer row dims, the two
// halves (stride D/2) and the batch. A box {D/2, ti, to, 2, 1} therefore lands
// in shared memory as [half][outer][inner][D/2] -- the tile's first halves,
// then its second halves -- so the lanes of a quarter warp, which read the
// same half of consecutive rows, read 128 contiguous bytes (no bank conflicts).
struct alignas(64) TmaTensor {
  CUtensorMap map;
};

struct TmaFwdArgs {
  TmaTensor in[2];      // q, k
  TmaTensor out_map[2]; // q_out, k_out as TMA store targets (when store_tma)
  int store_tma;        // 1: outputs staged in the stage's q / k tiles and stored by TMA
  void* out[2];         // q_out, k_out
  RowStrides so[2];
  const float* w;
  const float* scales;
  const float* sin;
  const float* cos;
  int64_t sin_b, cos_b;  // batch strides of the tables; their n stride is D/2
  float* rms[2];         // optional: r per row, FP32 [B, H, N]
  int64_t B, N;
  int H;
  float eps;
  TmaPlan p;
};

struct TmaBwdArgs {
  TmaTensor in[4];      // q, grad_q_out, k, grad_k_out
  TmaTensor out[2];     // dq, dk as TMA store targets (when store_tma)
  int store_tma;        // 1: dq / dk staged in the stage's q / k tiles and stored by TMA
  void* dx[2];          // dq, dk
  RowStrides sd[2];
  const float* w;
  const float* scales;
  const float* sin;
  const float* cos;
  int64_t sin_b, cos_b;
  float* partials;      // [grid, 2*D + H]
  const float* rms[2];  // inverse backward: saved r per row (in[] hold q_out, k_out)
  int64_t B, N;
  int H;
  float eps;
  TmaPlan p;
};

TmaPlan plan_tma(int64_t B, int64_t H, int64_t N, int D, int dtype, bool heads_inner, int stages);
size_t tma_smem_bytes(const TmaPlan& p, int D, int n_tensors, int H, bool inv = false);
// Read (synchronously) and optionally clear the error words of the TMA
// prologue kernels, of the fused QKV GEMM and of its backward GEMMs.
cudaError_t read_device_error(int* value, bool reset);
cudaError_t read_gemm_device_error(int* value, bool reset);
cudaError_t read_gemm_bwd_device_error(int* value, bool reset);
cudaError_t read_peer_device_error(int* value, bool reset);
// One thread waits (bounded by `tries` polls) on a barrier nothing arrives at.
cudaError_t launch_selftest_wait_timeout(uint32_t tries, cudaStream_t stream);
int64_t tma_grid(bool bwd, const TmaPlan& p, int H, int D, int dtype, bool inv = false);
cudaError_t launch_fwd_tma(const TmaFwdArgs& a, int dtype, int D, cudaStream_t stream);
struct BwdReduce;
cudaError_t launch_bwd_tma(const TmaBwdArgs& a, float* dw, float* ds, int dtype, int D,
                           bool inv, const BwdReduce& red, cudaStream_t stream);

// ---------------------------------------------------------------------------
// Geometry of a problem (layout-dependent, device-independent).
Geometry plan_geometry(int64_t B, int64_t H, int64_t N, int D, bool heads_inner);

// Persistent grid for a kernel: min(items, SMs x resident CTAs per SM).
int64_t persistent_grid(const void* kernel, size_t smem_bytes, int64_t n_items,
                        int threads = kThreads);

// Fixed-order sum of the [G, C] per-CTA partials into dw [two_d] and ds [C - two_d].
cudaError_t launch_bwd_finalize(const float* partials, int64_t G, int C, int two_d, float* dw,
                                float* ds, cudaStream_t stream);

// Where the backward's per-CTA partials go: the local fixed-order sum (peers
// null), or that sum added over the ranks of a peer group in one kernel
// (peer_reduce.cu).
struct BwdReduce {
  const flash_prologue_peers* peers = nullptr;
  uint32_t epoch = 0;
};
cudaError_t launch_bwd_reduce(const float* partials, int64_t G, int C, int two_d, float* dw, float* ds,
                              const BwdReduce& red, cudaStream_t stream);

// Launchers; return a cudaError_t from the launch.
cudaError_t launch_fwd(const FwdArgs& a, int dtype, int D, bool vec, cudaStream_t stream);

// Grid the backward kernel uses for this geometry on the current device.
// `inv` selects the inverse backward (rows rebuilt from outputs and saved r).
int64_t bwd_grid(const Geometry& g, int H, int D, int dtype, bool vec, bool inv = false);
size_t bwd_smem_bytes(int H, int D, bool inv = false);
cudaError_t launch_bwd(const BwdArgs& a, float* dw, float* ds, int dtype, int D, bool vec,
                       bool inv, const BwdReduce& red, cudaStream_t stream);

}  // namespace flash_prologue
