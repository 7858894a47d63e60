// Forward prologue kernel: per-head RMSNorm of Q and K, split-half RoPE, Q
// scaled by exp(scales[h]), one cast to the activation dtype.
//
// Arithmetic follows the reference formulation flash_attn_prologue/functional.py:89-94
// (x.float(); x * rsqrt(mean(x^2) + eps) * w; cat(a*cos - b*sin, b*cos + a*sin);
// Q * exp(scale); .to(dtype)) operation by operation, with every product and sum
// rounded separately (no FMA contraction) so the FP32 intermediates round like
// the eager formulation; only the order of the D-element sum of squares differs.
// Optionally the kernel also stores r = 1/sqrt(mean(x^2)+eps) of every row (the
// saved statistic of the inverse formulation, fused_epilogue.py:1916-1917).
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

  Cursor4 cur;
  for (cur.init(blockIdx.x, a.g.radix); cur.d[3] < a.B; cur.advance(a.g.radix)) {
    const int t = (int)cur.d[0];
    const int64_t pb = cur.d[1], hg = cur.d[2], b = cur.d[3];
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
      const float ss = row_sum<L>(lane_sumsq(x1, x2));
      if (!ok) continue;  // after the shuffles: every lane took part in them
      const float r = inv_rms<D>(ss, a.eps);
      if (a.rms[t] != nullptr && c == 0) a.rms[t][(b * a.H + h) * a.N + n] = r;
      Chunk<T> out1, out2;
      fwd_lane(x1, x2, r, w + j0, w + HALF + j0, sn, cs, t == 0, t == 0 ? e_s[h] : 1.f, out1, out2);
      T* yp = yb + b * sy.b + (int64_t)h * sy.h + n * sy.n + j0;
      store_stream<T, VEC>(yp, out1);
      store_stream<T, VEC>(yp + HALF, out2);
    }
  }
}

template <typename T, int D, bool VEC>
static cudaError_t launch_fwd_t(const FwdArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)(2 * D + a.H) * sizeof(float);
  const void* fn = reinterpret_cast<const void*>(&prologue_fwd_kernel<T, D, VEC>);
  const int64_t grid = persistent_grid(fn, smem, a.g.n_items);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  FwdArgs args = a;
  args.g.radix = make_radix(2, a.g.n_pos_blocks, a.g.n_head_groups, grid);
  return launch_kernel(prologue_fwd_kernel<T, D, VEC>, dim3((unsigned)grid), dim3(kThreads), smem, stream,
                       args);
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
