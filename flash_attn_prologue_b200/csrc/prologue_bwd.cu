// Backward prologue: dq, dk and the weight / log-scale gradients in one pass
// over q, k, grad_q_out, grad_k_out, followed by a small fixed-order reduction.
//
// Per row (x = q or k, g = upstream gradient, e = exp(scales[h]) for Q, 1 for K),
// the identities of the reference backward (flash_attn_prologue/fused_epilogue.py:1047-1126):
//   r  = rsqrt(mean(x^2)+eps),  n = x*r
//   g' = g*e
//   dn_j = g'_j cos_j + g'_{j+D/2} sin_j,  dn_{j+D/2} = g'_{j+D/2} cos_j - g'_j sin_j
//   d scales[h]   += sum_j g'_j * rot(n*w)_j  =  sum_j dn_j w_j n_j   (Q rows only;
//                    the rotation is orthogonal, so the reference's separate dot
//                    product equals the one dx needs anyway)
//   d w[t][j]     += dn_j * n_j
//   dx_j = r * (dn_j w_j - n_j * sum_i(dn_i w_i n_i) / D)
// evaluated with e folded into r (bwd_lane_reduce / lane_dx): with
// d0 = R^T g, re = r e and n' = x re, dn = e d0, d w += d0 n', the row sum is
// sum_i d0_i w_i n'_i, and dx = re (d0 w) - n' (r sum / D) / e.
// The reference accumulates the two parameter gradients with float atomics
// (fused_epilogue.py:1129-1207), whose order changes run to run. Here every
// CTA owns fixed rows (persistent, round-robin items); its threads keep
// register/shared partials that are combined in a fixed order into one
// [2*D + H] partial per CTA, and a second kernel sums the CTA partials in CTA
// order. The result is bit-identical on every run with the same grid.
//
// INV = true is the inverse backward (fused_epilogue.py:2200-2300): x[] hold the
// forward outputs and rms[] the saved r of every row; the normalised row n is
// rebuilt from them (inv_lane_reduce) instead of being recomputed from q and k.
#include "prologue_host.h"

namespace flash_prologue {

template <typename T, int D, bool VEC, bool INV>
__global__ void __launch_bounds__(kThreads) prologue_bwd_kernel(const BwdArgs a) {
  constexpr int L = D / 16;
  constexpr int HALF = D / 2;
  constexpr int LOG2_L = (L == 2) ? 1 : (L == 4) ? 2 : (L == 8) ? 3 : 4;
  extern __shared__ float smem[];
  // w and 1 / w are read as float pairs (8-byte loads), so they come first,
  // at even offsets; the H-sized arrays, whose length may be odd, follow.
  float* w_s = smem;                          // [2 * D]
  float* iw_s = w_s + 2 * D;                  // INV: [2 * D] 1 / w
  float* e_s = iw_s + (INV ? 2 * D : 0);      // [H]
  float* ds_s = e_s + a.H;                    // [kWarps][H]
  float* dw_s = ds_s + kWarps * a.H;          // [kWarps][D]
  float* ie_s = dw_s + kWarps * D;            // INV: [H] 1 / exp(scales)
  for (int i = threadIdx.x; i < 2 * D; i += kThreads) w_s[i] = a.w[i];
  for (int i = threadIdx.x; i < a.H; i += kThreads) e_s[i] = (float)exp((double)a.scales[i]);
  for (int i = threadIdx.x; i < kWarps * a.H; i += kThreads) ds_s[i] = 0.f;
  if constexpr (INV) {
    for (int i = threadIdx.x; i < 2 * D; i += kThreads) iw_s[i] = __frcp_rn(a.w[i]);
    for (int i = threadIdx.x; i < a.H; i += kThreads) ie_s[i] = (float)(1.0 / exp((double)a.scales[i]));
  }
  __syncthreads();

  // The host makes the grid even (or equal to the even item count), so every
  // item of this CTA has the tensor index of its first item.
  const int t = blockIdx.x & 1;
  const T* xb = static_cast<const T*>(a.x[t]);
  const T* gb = static_cast<const T*>(a.gy[t]);
  T* db = static_cast<T*>(a.dx[t]);
  const RowStrides sx = a.sx[t], sg = a.sgy[t], sd = a.sdx[t];
  const float* w = w_s + t * D;
  const float* iw = iw_s + t * D;
  const float* rms = INV ? a.rms[t] : nullptr;

  int c, hs, ps;
  thread_slots(a.g, threadIdx.x, c, hs, ps);
  const int HS = 1 << a.g.log2_hs;
  const int PS = 1 << a.g.log2_ps;
  const int heads_per_item = a.g.hi * HS;
  const int j0 = c * kChunk;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;

  // Lane bits (within the warp) that select a position slot: lanes that differ
  // only in these bits and in the chunk bits hold rows of the same head.
  const int warp_slot_bits = 5 - LOG2_L;
  int ps_lo, ps_hi;  // ps bits occupy lane bits [ps_lo, ps_hi)
  if (a.g.heads_inner) {
    ps_lo = LOG2_L + min(a.g.log2_hs, warp_slot_bits);
    ps_hi = 5;
  } else {
    ps_lo = LOG2_L;
    ps_hi = LOG2_L + min(a.g.log2_ps, warp_slot_bits);
  }
  const bool ds_writer = (lane & ((1 << ps_hi) - 1) & ~((1 << ps_lo) - 1)) == 0 && c == 0;

  float2 acc1p[kPairs], acc2p[kPairs];  // d w partials for elements j0.. and HALF+j0..
#pragma unroll
  for (int q = 0; q < kPairs; ++q) { acc1p[q] = make_float2(0.f, 0.f); acc2p[q] = make_float2(0.f, 0.f); }

  Cursor4 cur;
  for (cur.init(blockIdx.x, a.g.radix); cur.d[3] < a.B; cur.advance(a.g.radix)) {
    const int64_t pb = cur.d[1], hg = cur.d[2], b = cur.d[3];
    const int64_t n = pb * PS + ps;
    const bool pos_ok = n < a.N;

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
      Chunk<T> x1, x2, g1, g2;
      if (ok) {
        const T* xp = xb + b * sx.b + (int64_t)h * sx.h + n * sx.n + j0;
        const T* gp = gb + b * sg.b + (int64_t)h * sg.h + n * sg.n + j0;
        load_stream<T, VEC>(x1, xp);
        load_stream<T, VEC>(x2, xp + HALF);
        load_stream<T, VEC>(g1, gp);
        load_stream<T, VEC>(g2, gp + HALF);
      } else {
#pragma unroll
        for (int k = 0; k < Chunk<T>::kWords; ++k) { x1.w[k] = 0; x2.w[k] = 0; g1.w[k] = 0; g2.w[k] = 0; }
      }
      const float e = (t == 0 && h < a.H) ? e_s[h] : 1.f;
      float2 dnw1[kPairs], dnw2[kPairs];  // u = d0 w (INV: t = d0 w)
      float2 n1[kPairs], n2[kPairs];      // n' = e n: x re, or rebuilt from the outputs (INV)
      float r, re, dsum;
      if constexpr (INV) {
        r = ok ? __ldg(rms + (b * a.H + h) * a.N + n) : 0.f;
        re = __fmul_rn(r, e);
        float part = 0.f;
        if (ok) {
          part = inv_lane_reduce(x1, x2, g1, g2, w + j0, w + HALF + j0, iw + j0, iw + HALF + j0, sn,
                                 cs, acc1p, acc2p, n1, n2, dnw1, dnw2);
        }
        dsum = row_sum<L>(part);
      } else {
        r = inv_rms_bwd<D>(row_sum<L>(lane_sumsq2(x1, x2)), a.eps);
        re = __fmul_rn(r, e);
        dsum = row_sum<L>(bwd_lane_reduce(x1, x2, g1, g2, re, w + j0, w + HALF + j0, sn, cs, acc1p,
                                          acc2p, dnw1, dnw2, n1, n2));
      }
      if (t == 0) {
        // d scales: the row's sum(dn w n), reduced over the warp's position slots.
        float v = dsum;
        for (int bit = ps_lo; bit < ps_hi; ++bit)
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1 << bit));
        if (ds_writer && h < a.H) ds_s[warp * a.H + h] += v;
      }
      if (!ok) continue;
      Chunk<T> out1, out2;
      if constexpr (INV)
        lane_dx<T>(n1, n2, dnw1, dnw2, re,
                       __fmul_rn(__fmul_rn(r, dsum * (1.0f / (float)D)), t == 0 ? ie_s[h] : 1.f),
                       out1, out2);
      else
        lane_dx<T>(n1, n2, dnw1, dnw2, re, __fdividef(__fmul_rn(r, dsum * (1.0f / (float)D)), e), out1,
                   out2);
      T* dp = db + b * sd.b + (int64_t)h * sd.h + n * sd.n + j0;
      store_stream<T, VEC>(dp, out1);
      store_stream<T, VEC>(dp + HALF, out2);
    }
  }

  // d w: combine lanes that hold the same chunk (fixed xor order), then warps.
  float acc1[kChunk], acc2[kChunk];
  unpair(acc1p, acc1);
  unpair(acc2p, acc2);
#pragma unroll
  for (int j = 0; j < kChunk; ++j) {
#pragma unroll
    for (int o = L; o < 32; o <<= 1) {
      acc1[j] = __fadd_rn(acc1[j], __shfl_xor_sync(0xffffffffu, acc1[j], o));
      acc2[j] = __fadd_rn(acc2[j], __shfl_xor_sync(0xffffffffu, acc2[j], o));
    }
  }
  if (lane < L) {
    float* dst = dw_s + warp * D;
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      dst[j0 + j] = acc1[j];
      dst[HALF + j0 + j] = acc2[j];
    }
  }
  __syncthreads();
  const int C = 2 * D + a.H;
  float* out = a.partials + (int64_t)blockIdx.x * C;
  for (int col = threadIdx.x; col < C; col += kThreads) {
    float v = 0.f;
    if (col < 2 * D) {
      if ((col >= D) == (t == 1)) {
        const int j = col - t * D;
#pragma unroll
        for (int w8 = 0; w8 < kWarps; ++w8) v = __fadd_rn(v, dw_s[w8 * D + j]);
      }
    } else if (t == 0) {
#pragma unroll
      for (int w8 = 0; w8 < kWarps; ++w8) v = __fadd_rn(v, ds_s[w8 * a.H + (col - 2 * D)]);
    }
    out[col] = v;
  }
}

// Sums the [G, C] CTA partials over G in a fixed order: warp w of CTA x sums
// rows w, w+8, ... of 32 columns; the 8 warp sums are then added in warp order.
__global__ void __launch_bounds__(kThreads) prologue_bwd_finalize_kernel(
    const float* __restrict__ partials, int64_t G, int C, int two_d, float* __restrict__ dw,
    float* __restrict__ ds) {
  __shared__ float part[kWarps][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  const float v = col < C ? strided_column_sum(partials, G, C, col, warp, kWarps) : 0.f;
  part[warp][lane] = v;
  __syncthreads();
  if (warp == 0 && col < C) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s = __fadd_rn(s, part[w][lane]);
    if (col < two_d) dw[col] = s;
    else ds[col - two_d] = s;
  }
}

size_t bwd_smem_bytes(int H, int D, bool inv) {
  return (size_t)(2 * D + H + kWarps * H + kWarps * D + (inv ? 2 * D + H : 0)) * sizeof(float);
}

// Grid for the backward kernel: persistent, and even whenever it is smaller
// than the (always even) item count, so each CTA sees a single tensor.
static int64_t even_grid(int64_t grid, int64_t n_items) {
  if (grid >= n_items) return n_items;
  return grid >= 2 ? (grid & ~int64_t(1)) : 2;
}

template <typename T, int D, bool VEC>
static const void* bwd_kernel_ptr(bool inv) {
  return inv ? reinterpret_cast<const void*>(&prologue_bwd_kernel<T, D, VEC, true>)
             : reinterpret_cast<const void*>(&prologue_bwd_kernel<T, D, VEC, false>);
}

static const void* bwd_kernel_for(int dtype, int D, bool vec, bool inv) {
#define FP_BWD_CASE(T)                                                                       \
  switch (D) {                                                                               \
    case 32: return vec ? bwd_kernel_ptr<T, 32, true>(inv) : bwd_kernel_ptr<T, 32, false>(inv);    \
    case 64: return vec ? bwd_kernel_ptr<T, 64, true>(inv) : bwd_kernel_ptr<T, 64, false>(inv);    \
    case 128: return vec ? bwd_kernel_ptr<T, 128, true>(inv) : bwd_kernel_ptr<T, 128, false>(inv); \
    case 256: return vec ? bwd_kernel_ptr<T, 256, true>(inv) : bwd_kernel_ptr<T, 256, false>(inv); \
    default: return nullptr;                                                                 \
  }
  switch (dtype) {
    case 0: FP_BWD_CASE(__nv_bfloat16)
    case 1: FP_BWD_CASE(__half)
    case 2: FP_BWD_CASE(float)
    default: return nullptr;
  }
#undef FP_BWD_CASE
}

int64_t bwd_grid(const Geometry& g, int H, int D, int dtype, bool vec, bool inv) {
  const void* fn = bwd_kernel_for(dtype, D, vec, inv);
  if (!fn) return -1;
  const int64_t grid = persistent_grid(fn, bwd_smem_bytes(H, D, inv), g.n_items);
  return grid > 0 ? even_grid(grid, g.n_items) : grid;
}

cudaError_t launch_bwd(const BwdArgs& a, float* dw, float* ds, int dtype, int D, bool vec,
                       bool inv, const BwdReduce& red, cudaStream_t stream) {
  const void* fn = bwd_kernel_for(dtype, D, vec, inv);
  if (!fn) return cudaErrorInvalidValue;
  const size_t smem = bwd_smem_bytes(a.H, D, inv);
  int64_t grid = persistent_grid(fn, smem, a.g.n_items);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  grid = even_grid(grid, a.g.n_items);
  BwdArgs launch_args = a;
  launch_args.g.radix = make_radix(2, a.g.n_pos_blocks, a.g.n_head_groups, grid);
  void* args[] = {&launch_args};
  cudaError_t err = cudaLaunchKernel(fn, dim3((unsigned)grid), dim3(kThreads), args, smem, stream);
  if (err != cudaSuccess) return err;
  return launch_bwd_reduce(a.partials, grid, 2 * D + a.H, 2 * D, dw, ds, red, stream);
}

cudaError_t launch_bwd_finalize(const float* partials, int64_t G, int C, int two_d, float* dw,
                                float* ds, cudaStream_t stream) {
  return launch_kernel(prologue_bwd_finalize_kernel, dim3((C + 31) / 32), dim3(kThreads), 0, stream,
                       partials, G, C, two_d, dw, ds);
}

}  // namespace flash_prologue
