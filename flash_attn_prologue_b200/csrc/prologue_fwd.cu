// Forward prologue kernel: per-head RMSNorm of Q and K, split-half RoPE, Q
// scaled by exp(scales[h]), one cast to the activation dtype.
//
// Arithmetic follows the reference formulation flash_attn_prologue/functional.py:89-94
// (x.float(); x * rsqrt(mean(x^2) + eps) * w; cat(a*cos - b*sin, b*cos + a*sin);
// Q * exp(scale); .to(dtype)) operation by operation, with every product and sum
// rounded separately (no FMA contraction) so the FP32 intermediates round like
// the eager formulation; only the order of the D-element sum of squares differs.
#include "prologue_host.h"

namespace flash_prologue {

template <typename T, int D, bool VEC>
__global__ void __launch_bounds__(kThreads) prologue_fwd_kernel(const FwdArgs a) {
  constexpr int L = D / 16;
  constexpr int HALF = D / 2;
  extern __shared__ float smem[];
  float* w_s = smem;           // [2 * D]
  float* e_s = smem + 2 * D;   // [H] exp(scales)
  for (int i = threadIdx.x; i < 2 * D; i += kThreads) w_s[i] = a.w[i];
  for (int i = threadIdx.x; i < a.H; i += kThreads) e_s[i] = (float)exp((double)a.scales[i]);
  __syncthreads();

  int c, hs, ps;
  thread_slots(a.g, threadIdx.x, c, hs, ps);
  const int HS = 1 << a.g.log2_hs;
  const int PS = 1 << a.g.log2_ps;
  const int heads_per_item = a.g.hi * HS;
  const int j0 = c * kChunk;

  for (int64_t item = blockIdx.x; item < a.g.n_items; item += gridDim.x) {
    int t;
    int64_t b, pb, hg;
    item_coords(a.g, item, t, b, pb, hg);
    const int64_t n = pb * PS + ps;
    const bool pos_ok = n < a.N;
    const T* xb = static_cast<const T*>(a.x[t]);
    T* yb = static_cast<T*>(a.y[t]);
    const RowStrides sx = a.sx[t], sy = a.sy[t];
    const float* w = w_s + t * D;

    float sn[kChunk], cs[kChunk];
    if (pos_ok) {
      load_table<VEC>(sn, a.sin + b * a.ssin.b + n * a.ssin.n + (int64_t)j0 * a.ssin.j, a.ssin.j);
      load_table<VEC>(cs, a.cos + b * a.scos.b + n * a.scos.n + (int64_t)j0 * a.scos.j, a.scos.j);
    } else {
#pragma unroll
      for (int j = 0; j < kChunk; ++j) { sn[j] = 0.f; cs[j] = 0.f; }
    }

    for (int i = 0; i < a.g.hi; ++i) {
      const int h = (int)hg * heads_per_item + i * HS + hs;
      const bool ok = pos_ok && h < a.H;
      Chunk<T> x1, x2;
      if (ok) {
        const T* xp = xb + b * sx.b + (int64_t)h * sx.h + n * sx.n + j0;
        load_stream<T, VEC>(x1, xp);
        load_stream<T, VEC>(x2, xp + HALF);
      } else {
#pragma unroll
        for (int k = 0; k < Chunk<T>::kWords; ++k) { x1.w[k] = 0; x2.w[k] = 0; }
      }

      // Sum of the rounded squares, lane-local then across the row's lanes.
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        const float u = chunk_get(x1, j);
        ss = __fadd_rn(ss, __fmul_rn(u, u));
      }
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        const float u = chunk_get(x2, j);
        ss = __fadd_rn(ss, __fmul_rn(u, u));
      }
      ss = row_sum<L>(ss);
      if (!ok) continue;  // after the shuffles: every lane took part in them

      const float r = inv_rms<D>(ss, a.eps);
      float o1[kChunk], o2[kChunk];
      // normed = (x * r) * w; rotate
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        const float y1 = __fmul_rn(__fmul_rn(chunk_get(x1, j), r), w[j0 + j]);
        const float y2 = __fmul_rn(__fmul_rn(chunk_get(x2, j), r), w[HALF + j0 + j]);
        o1[j] = __fsub_rn(__fmul_rn(y1, cs[j]), __fmul_rn(y2, sn[j]));
        o2[j] = __fadd_rn(__fmul_rn(y2, cs[j]), __fmul_rn(y1, sn[j]));
      }
      if (t == 0) {  // Q only: * exp(scale), after the rotation
        const float e = e_s[h];
#pragma unroll
        for (int j = 0; j < kChunk; ++j) { o1[j] = __fmul_rn(o1[j], e); o2[j] = __fmul_rn(o2[j], e); }
      }
      Chunk<T> out;
      T* yp = yb + b * sy.b + (int64_t)h * sy.h + n * sy.n + j0;
      chunk_set(out, o1);
      store_stream<T, VEC>(yp, out);
      chunk_set(out, o2);
      store_stream<T, VEC>(yp + HALF, out);
    }
  }
}

template <typename T, int D, bool VEC>
static cudaError_t launch_fwd_t(const FwdArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)(2 * D + a.H) * sizeof(float);
  const void* fn = reinterpret_cast<const void*>(&prologue_fwd_kernel<T, D, VEC>);
  const int64_t grid = persistent_grid(fn, smem, a.g.n_items);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  prologue_fwd_kernel<T, D, VEC><<<(unsigned)grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_fwd_d(const FwdArgs& a, bool vec, cudaStream_t stream) {
  return vec ? launch_fwd_t<T, D, true>(a, stream) : launch_fwd_t<T, D, false>(a, stream);
}

template <typename T>
static cudaError_t launch_fwd_dt(const FwdArgs& a, int D, bool vec, cudaStream_t stream) {
  switch (D) {
    case 32: return launch_fwd_d<T, 32>(a, vec, stream);
    case 64: return launch_fwd_d<T, 64>(a, vec, stream);
    case 128: return launch_fwd_d<T, 128>(a, vec, stream);
    case 256: return launch_fwd_d<T, 256>(a, vec, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_fwd(const FwdArgs& a, int dtype, int D, bool vec, cudaStream_t stream) {
  switch (dtype) {
    case 0: return launch_fwd_dt<__nv_bfloat16>(a, D, vec, stream);
    case 1: return launch_fwd_dt<__half>(a, D, vec, stream);
    case 2: return launch_fwd_dt<float>(a, D, vec, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace flash_prologue
