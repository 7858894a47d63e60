// Shared device helpers for the prologue kernels (forward, backward).
//
// Work decomposition used by both kernels
// ---------------------------------------
// A row is one (b, h, n) vector of D elements. Each thread owns one "chunk
// pair" of a row: elements [8c, 8c+8) of the first half and [D/2+8c, D/2+8c+8)
// of the second half, so the split-half RoPE partner of every element it holds
// is in the same thread (no shuffles for the rotation). L = D/16 lanes cover a
// row; sum-of-squares and dot products are reduced with L-lane xor butterflies,
// which give every lane of the group bit-identical results.
//
// A CTA of 256 threads has 256/L row slots, split into HS head slots x PS
// position slots. The slot order along lanes follows the smaller of the
// head/position strides of q ("heads inner" for packed [T,H,D] views,
// "positions inner" for dense [B,H,N,D]), so a warp's 16-byte accesses cover
// contiguous memory. A work item is (tensor t in {Q, K}, b, block of PS
// positions, group of HI*HS heads), with t the fastest index so the Q and K
// items of a position block run back to back and share its sin/cos rows in L2.
// The thread keeps its position's sin/cos chunk in registers and walks HI
// heads. CTAs are persistent and take items round-robin; with an even grid a
// CTA only ever sees one tensor.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace flash_prologue {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 8;  // elements per half-chunk owned by one lane

struct RowStrides {  // element strides of a [B, H, N, D] view (d stride is 1)
  int64_t b, h, n;
};
struct TableStrides {  // element strides of a sin/cos table indexed [b, n, j]
  int64_t b, n, j;
};

// Mixed-radix position of a persistent CTA's work item: digit 0 fastest,
// digit 3 unbounded. CTAs advance by the grid size without divisions: the
// digits of the grid size are precomputed on the host (make_radix).
struct Radix4 {
  int32_t ext[3];   // extents of digits 0..2
  int32_t step[4];  // digits of the grid size
};

struct Cursor4 {
  int32_t d[4];
  __device__ __forceinline__ void init(int32_t idx, const Radix4& r) {
    d[0] = idx % r.ext[0];
    idx /= r.ext[0];
    d[1] = idx % r.ext[1];
    idx /= r.ext[1];
    d[2] = idx % r.ext[2];
    d[3] = idx / r.ext[2];
  }
  __device__ __forceinline__ void advance(const Radix4& r) {
    d[0] += r.step[0];
    d[1] += r.step[1];
    d[2] += r.step[2];
    d[3] += r.step[3];
    if (d[0] >= r.ext[0]) { d[0] -= r.ext[0]; ++d[1]; }
    if (d[1] >= r.ext[1]) { d[1] -= r.ext[1]; ++d[2]; }
    if (d[2] >= r.ext[2]) { d[2] -= r.ext[2]; ++d[3]; }
  }
};

// Digits of `stride` in the radix (e0, e1, e2, unbounded). Every extent and
// the stride are below 2^31 (checked by the C-ABI layer).
inline Radix4 make_radix(int64_t e0, int64_t e1, int64_t e2, int64_t stride) {
  Radix4 r;
  r.ext[0] = (int32_t)e0; r.ext[1] = (int32_t)e1; r.ext[2] = (int32_t)e2;
  r.step[0] = (int32_t)(stride % e0); stride /= e0;
  r.step[1] = (int32_t)(stride % e1); stride /= e1;
  r.step[2] = (int32_t)(stride % e2);
  r.step[3] = (int32_t)(stride / e2);
  return r;
}

// Launch geometry shared by host planning and kernels.
struct Geometry {
  int log2_l;          // lanes per row = D / 16
  int log2_hs;         // head slots per CTA iteration
  int log2_ps;         // position slots per CTA iteration
  int heads_inner;     // 1: slot = hs + HS * ps, 0: slot = ps + PS * hs
  int hi;              // head iterations per item
  int64_t n_pos_blocks;
  int64_t n_head_groups;
  int64_t n_items;     // 2 (tensors) * B * n_head_groups * n_pos_blocks
  Radix4 radix;        // digits (tensor, position block, head group) + batch
};

// ---------------------------------------------------------------------------
// 8-element chunks of the activation dtype, kept as raw 32-bit words.
template <typename T>
struct Chunk {
  static constexpr int kWords = kChunk * sizeof(T) / 4;
  uint32_t w[kWords];
};

template <typename T>
__device__ __forceinline__ float chunk_get(const Chunk<T>& c, int i);

template <>
__device__ __forceinline__ float chunk_get<__nv_bfloat16>(const Chunk<__nv_bfloat16>& c, int i) {
  const uint32_t word = c.w[i >> 1];
  return __uint_as_float((i & 1) ? (word & 0xffff0000u) : (word << 16));
}
template <>
__device__ __forceinline__ float chunk_get<__half>(const Chunk<__half>& c, int i) {
  const uint32_t word = c.w[i >> 1];
  const unsigned short bits = (i & 1) ? (unsigned short)(word >> 16) : (unsigned short)(word & 0xffffu);
  return __half2float(__ushort_as_half(bits));
}
template <>
__device__ __forceinline__ float chunk_get<float>(const Chunk<float>& c, int i) {
  return __uint_as_float(c.w[i]);
}

// Round-to-nearest-even cast of 8 floats into a chunk.
template <typename T>
__device__ __forceinline__ void chunk_set(Chunk<T>& c, const float (&v)[kChunk]);

template <>
__device__ __forceinline__ void chunk_set<__nv_bfloat16>(Chunk<__nv_bfloat16>& c, const float (&v)[kChunk]) {
#pragma unroll
  for (int i = 0; i < kChunk / 2; ++i) {
    __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    c.w[i] = *reinterpret_cast<uint32_t*>(&p);
  }
}
template <>
__device__ __forceinline__ void chunk_set<__half>(Chunk<__half>& c, const float (&v)[kChunk]) {
#pragma unroll
  for (int i = 0; i < kChunk / 2; ++i) {
    __half2 p = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    c.w[i] = *reinterpret_cast<uint32_t*>(&p);
  }
}
template <>
__device__ __forceinline__ void chunk_set<float>(Chunk<float>& c, const float (&v)[kChunk]) {
#pragma unroll
  for (int i = 0; i < kChunk; ++i) c.w[i] = __float_as_uint(v[i]);
}

// Streaming (evict-first) load of a chunk. VEC: 16-byte accesses; otherwise
// element-wise accesses for views whose rows are not 16-byte aligned.
template <typename T, bool VEC>
__device__ __forceinline__ void load_stream(Chunk<T>& c, const T* p) {
  if constexpr (VEC) {
    const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < Chunk<T>::kWords / 4; ++i) {
      uint4 v = __ldcs(p4 + i);
      c.w[4 * i + 0] = v.x; c.w[4 * i + 1] = v.y; c.w[4 * i + 2] = v.z; c.w[4 * i + 3] = v.w;
    }
  } else {
    if constexpr (sizeof(T) == 4) {
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(p);
#pragma unroll
      for (int i = 0; i < kChunk; ++i) c.w[i] = pw[i];
    } else {
      const unsigned short* ph = reinterpret_cast<const unsigned short*>(p);
#pragma unroll
      for (int i = 0; i < kChunk / 2; ++i)
        c.w[i] = (uint32_t)ph[2 * i] | ((uint32_t)ph[2 * i + 1] << 16);
    }
  }
}

// Store of a chunk. VEC: 16-byte stores with the default write-back policy
// (the streaming .cs hint measured slightly slower on the TMA kernels).
template <typename T, bool VEC>
__device__ __forceinline__ void store_stream(T* p, const Chunk<T>& c) {
  if constexpr (VEC) {
    uint4* p4 = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < Chunk<T>::kWords / 4; ++i)
      p4[i] = make_uint4(c.w[4 * i + 0], c.w[4 * i + 1], c.w[4 * i + 2], c.w[4 * i + 3]);
  } else {
    if constexpr (sizeof(T) == 4) {
      uint32_t* pw = reinterpret_cast<uint32_t*>(p);
#pragma unroll
      for (int i = 0; i < kChunk; ++i) pw[i] = c.w[i];
    } else {
      unsigned short* ph = reinterpret_cast<unsigned short*>(p);
#pragma unroll
      for (int i = 0; i < kChunk / 2; ++i) {
        ph[2 * i] = (unsigned short)(c.w[i] & 0xffffu);
        ph[2 * i + 1] = (unsigned short)(c.w[i] >> 16);
      }
    }
  }
}

// 8 FP32 sin or cos values for one (b, n) and chunk, read through the
// read-only path (the tables are reused by every head of a position).
template <bool VEC>
__device__ __forceinline__ void load_table(float (&v)[kChunk], const float* p, int64_t sj) {
  if constexpr (VEC) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
    float4 a = __ldg(p4), b = __ldg(p4 + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < kChunk; ++i) v[i] = __ldg(p + i * sj);
  }
}

// Sum over the L lanes of a row (xor butterfly: every lane gets the same bits).
template <int L>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int o = 1; o < L; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 1 / sqrt(mean + eps) with an IEEE-rounded sqrt and an IEEE-rounded
// reciprocal (the rounding the CPU formulation 1/sqrt(x) gets). D is a power of
// two, so mean = sum * (1/D) is exactly sum / D.
template <int D>
__device__ __forceinline__ float inv_rms(float sumsq, float eps) {
  static_assert((D & (D - 1)) == 0, "head dim must be a power of two");
  const float mean = __fmul_rn(sumsq, 1.0f / (float)D);
  return __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
}

// The backward's recomputed r: the hardware reciprocal square root
// (rsqrt.approx.f32, relative error below 2^-22), as the reference's CuTe
// backward recomputes its per-row rstd (cute.math.rsqrt,
// flash_attn_prologue/fused_epilogue.py:1055-1056). Gradients carry a
// tolerance, so the backward does not pay for the IEEE-rounded sequence.
template <int D>
__device__ __forceinline__ float inv_rms_bwd(float sumsq, float eps) {
  static_assert((D & (D - 1)) == 0, "head dim must be a power of two");
  return rsqrtf(__fadd_rn(__fmul_rn(sumsq, 1.0f / (float)D), eps));
}

// ---------------------------------------------------------------------------
// Per-row arithmetic shared by the register-path and the TMA kernels (so
// both give bit-identical results). A lane holds the chunk pair
// x1 = x[j0 .. j0+8), x2 = x[D/2+j0 .. D/2+j0+8) of its row and works on
// element pairs (2p, 2p+1) with sm_100's paired FP32 instructions
// (__fmul2_rn / __fadd2_rn / __ffma2_rn): each half rounds exactly like the
// scalar IEEE operation, at half the instruction count.
constexpr int kPairs = kChunk / 2;

template <typename T>
__device__ __forceinline__ float2 chunk_get2(const Chunk<T>& c, int p);

template <>
__device__ __forceinline__ float2 chunk_get2<__nv_bfloat16>(const Chunk<__nv_bfloat16>& c, int p) {
  const uint32_t word = c.w[p];
  return make_float2(__uint_as_float(word << 16), __uint_as_float(word & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 chunk_get2<__half>(const Chunk<__half>& c, int p) {
  const uint32_t word = c.w[p];
  return __half22float2(*reinterpret_cast<const __half2*>(&word));
}
template <>
__device__ __forceinline__ float2 chunk_get2<float>(const Chunk<float>& c, int p) {
  return make_float2(__uint_as_float(c.w[2 * p]), __uint_as_float(c.w[2 * p + 1]));
}

template <typename T>
__device__ __forceinline__ void chunk_set2(Chunk<T>& c, const float2 (&v)[kPairs]) {
  float f[kChunk];
#pragma unroll
  for (int p = 0; p < kPairs; ++p) { f[2 * p] = v[p].x; f[2 * p + 1] = v[p].y; }
  chunk_set(c, f);
}

__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 neg2(float2 v) { return make_float2(-v.x, -v.y); }
__device__ __forceinline__ float2 ld_pair(const float* p, int q) {
  return reinterpret_cast<const float2*>(p)[q];
}

// Lane-partial sum of squares over two interleaved pair accumulators. For
// 16-bit inputs x*x is exact in FP32, so the fused multiply-add rounds exactly
// like "square, then add"; FP32 inputs square and add separately.
template <typename T>
__device__ __forceinline__ float lane_sumsq(const Chunk<T>& x1, const Chunk<T>& x2) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    const float2 u = chunk_get2(x1, p);
    acc = (sizeof(T) == 2) ? __ffma2_rn(u, u, acc) : __fadd2_rn(acc, __fmul2_rn(u, u));
  }
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    const float2 u = chunk_get2(x2, p);
    acc = (sizeof(T) == 2) ? __ffma2_rn(u, u, acc) : __fadd2_rn(acc, __fmul2_rn(u, u));
  }
  return __fadd_rn(acc.x, acc.y);
}

// lane_sumsq with the two halves summed in independent chains (backward only:
// its r carries no bit-parity requirement, and the shorter chain hides latency).
template <typename T>
__device__ __forceinline__ float lane_sumsq2(const Chunk<T>& x1, const Chunk<T>& x2) {
  float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    const float2 u = chunk_get2(x1, p), v = chunk_get2(x2, p);
    a = (sizeof(T) == 2) ? __ffma2_rn(u, u, a) : __fadd2_rn(a, __fmul2_rn(u, u));
    b = (sizeof(T) == 2) ? __ffma2_rn(v, v, b) : __fadd2_rn(b, __fmul2_rn(v, v));
  }
  const float2 s = __fadd2_rn(a, b);
  return __fadd_rn(s.x, s.y);
}

// Forward outputs of one lane: normed = (x * r) * w, rotated, times e for Q.
// Every product and sum rounds separately, as in the eager formulation
// (a - b is computed as a + (-b), which rounds identically).
template <typename T>
__device__ __forceinline__ void fwd_lane(const Chunk<T>& x1, const Chunk<T>& x2, float r,
                                         const float* wa, const float* wb, const float (&sn)[kChunk],
                                         const float (&cs)[kChunk], bool scale, float e,
                                         Chunk<T>& out1, Chunk<T>& out2) {
  const float2 r2 = splat2(r), e2 = splat2(e);
  float2 o1[kPairs], o2[kPairs];
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    const float2 c2 = make_float2(cs[2 * p], cs[2 * p + 1]);
    const float2 s2 = make_float2(sn[2 * p], sn[2 * p + 1]);
    const float2 y1 = __fmul2_rn(__fmul2_rn(chunk_get2(x1, p), r2), ld_pair(wa, p));
    const float2 y2 = __fmul2_rn(__fmul2_rn(chunk_get2(x2, p), r2), ld_pair(wb, p));
    o1[p] = __fadd2_rn(__fmul2_rn(y1, c2), neg2(__fmul2_rn(y2, s2)));
    o2[p] = __fadd2_rn(__fmul2_rn(y2, c2), __fmul2_rn(y1, s2));
    if (scale) {
      o1[p] = __fmul2_rn(o1[p], e2);
      o2[p] = __fmul2_rn(o2[p], e2);
    }
  }
  chunk_set2(out1, o1);
  chunk_set2(out2, o2);
}

// Backward, reduction part of one lane. With d0 = R^T g (the inverse rotation
// of the upstream gradient, without the Q scale e) and re = r * e (r for K):
// dy = e d0 is the gradient of the normed row n w and dn = dy w = e u with
// u = d0 w, so
//   d w partial:  acc += d0 * (x re)                        (= dy n)
//   returned:     lane partial of sum_j u_j (x_j re)        (= <dn, n>)
// and u is kept for the dx part. The returned sum is also the row's
// contribution to d scale: <dn, n> = <R^T g', n w> = <g', R(n w)> =
// sum_j dq_out_j q_out_j. The lane keeps n' = x re for the dx part (lane_dx),
// so x is not unpacked again. Two independent partial sums (first / second
// half) shorten the dependency chain.
template <typename T>
__device__ __forceinline__ float bwd_lane_reduce(const Chunk<T>& x1, const Chunk<T>& x2,
                                                 const Chunk<T>& g1, const Chunk<T>& g2, float re,
                                                 const float* wa, const float* wb,
                                                 const float (&sn)[kChunk], const float (&cs)[kChunk],
                                                 float2 (&acc1)[kPairs], float2 (&acc2)[kPairs],
                                                 float2 (&u1)[kPairs], float2 (&u2)[kPairs],
                                                 float2 (&nx1)[kPairs], float2 (&nx2)[kPairs]) {
  const float2 re2 = splat2(re);
  float2 ds1 = make_float2(0.f, 0.f), ds2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    const float2 c2 = make_float2(cs[2 * p], cs[2 * p + 1]);
    const float2 s2 = make_float2(sn[2 * p], sn[2 * p + 1]);
    const float2 ga = chunk_get2(g1, p), gb = chunk_get2(g2, p);
    const float2 d1 = __ffma2_rn(ga, c2, __fmul2_rn(gb, s2));
    const float2 d2 = __ffma2_rn(gb, c2, neg2(__fmul2_rn(ga, s2)));
    const float2 n1 = __fmul2_rn(chunk_get2(x1, p), re2);
    const float2 n2 = __fmul2_rn(chunk_get2(x2, p), re2);
    nx1[p] = n1;
    nx2[p] = n2;
    acc1[p] = __ffma2_rn(d1, n1, acc1[p]);
    acc2[p] = __ffma2_rn(d2, n2, acc2[p]);
    u1[p] = __fmul2_rn(d1, ld_pair(wa, p));
    u2[p] = __fmul2_rn(d2, ld_pair(wb, p));
    ds1 = __ffma2_rn(u1[p], n1, ds1);
    ds2 = __ffma2_rn(u2[p], n2, ds2);
  }
  const float2 ds = __fadd2_rn(ds1, ds2);
  return __fadd_rn(ds.x, ds.y);
}

// ---------------------------------------------------------------------------
// Inverse backward (the outputs and r are saved instead of the inputs; the
// reference's qknorm_rope_scale_cute_inverse_backward,
// flash_attn_prologue/fused_epilogue.py:2200-2300). The forward output of a row
// is o = e R(n w), so m0 = R^T o = e n w and n' = m0 / w = e n (1/w is the
// precomputed reciprocal iw). With d0 = R^T g, the gradient of n w is
// dy = e d0, so
//   d w partial:  acc += d0 * n'                       (= dy n)
//   returned:     lane partial of sum_j d0_j m0_j      (= <dy w, n> = <dn, n>, and
//                 <R^T g, R^T o> = sum_j dq_out_j q_out_j: the d scale term)
// The lane keeps n' and t = d0 w for the dx part. Two independent partial sums
// (first / second half) shorten the dependency chain.
template <typename T>
__device__ __forceinline__ float inv_lane_reduce(const Chunk<T>& o1, const Chunk<T>& o2,
                                                 const Chunk<T>& g1, const Chunk<T>& g2,
                                                 const float* wa, const float* wb, const float* iwa,
                                                 const float* iwb, const float (&sn)[kChunk],
                                                 const float (&cs)[kChunk], float2 (&acc1)[kPairs],
                                                 float2 (&acc2)[kPairs], float2 (&np1)[kPairs],
                                                 float2 (&np2)[kPairs], float2 (&t1)[kPairs],
                                                 float2 (&t2)[kPairs]) {
  float2 ds1 = make_float2(0.f, 0.f), ds2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    const float2 c2 = make_float2(cs[2 * p], cs[2 * p + 1]);
    const float2 s2 = make_float2(sn[2 * p], sn[2 * p + 1]);
    const float2 oa = chunk_get2(o1, p), ob = chunk_get2(o2, p);
    const float2 ga = chunk_get2(g1, p), gb = chunk_get2(g2, p);
    const float2 m1 = __ffma2_rn(oa, c2, __fmul2_rn(ob, s2));
    const float2 m2 = __ffma2_rn(ob, c2, neg2(__fmul2_rn(oa, s2)));
    const float2 d1 = __ffma2_rn(ga, c2, __fmul2_rn(gb, s2));
    const float2 d2 = __ffma2_rn(gb, c2, neg2(__fmul2_rn(ga, s2)));
    np1[p] = __fmul2_rn(m1, ld_pair(iwa, p));
    np2[p] = __fmul2_rn(m2, ld_pair(iwb, p));
    acc1[p] = __ffma2_rn(d1, np1[p], acc1[p]);
    acc2[p] = __ffma2_rn(d2, np2[p], acc2[p]);
    t1[p] = __fmul2_rn(d1, ld_pair(wa, p));
    t2[p] = __fmul2_rn(d2, ld_pair(wb, p));
    ds1 = __ffma2_rn(d1, m1, ds1);
    ds2 = __ffma2_rn(d2, m2, ds2);
  }
  const float2 ds = __fadd2_rn(ds1, ds2);
  return __fadd_rn(ds.x, ds.y);
}

// Backward (both formulations), dx of one lane: dx = r (dn - n m) with
// dn = e t (t = d0 w), n = n' / e (n' = e n: x re, or rebuilt from the outputs)
// and m = <dn, n> / D, evaluated as re * t - n' * kx with re = r e and
// kx = r m / e.
template <typename T>
__device__ __forceinline__ void lane_dx(const float2 (&np1)[kPairs], const float2 (&np2)[kPairs],
                                            const float2 (&t1)[kPairs], const float2 (&t2)[kPairs],
                                            float re, float kx, Chunk<T>& out1, Chunk<T>& out2) {
  const float2 re2 = splat2(re), nk2 = splat2(-kx);
  float2 o1[kPairs], o2[kPairs];
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    o1[p] = __ffma2_rn(np1[p], nk2, __fmul2_rn(re2, t1[p]));
    o2[p] = __ffma2_rn(np2[p], nk2, __fmul2_rn(re2, t2[p]));
  }
  chunk_set2(out1, o1);
  chunk_set2(out2, o2);
}

// Sum of a lane's two d w pair accumulators into 8 element values.
__device__ __forceinline__ void unpair(const float2 (&a)[kPairs], float (&v)[kChunk]) {
#pragma unroll
  for (int p = 0; p < kPairs; ++p) { v[2 * p] = a[p].x; v[2 * p + 1] = a[p].y; }
}

// Decompose a CTA thread into (chunk c, head slot hs, position slot ps).
__device__ __forceinline__ void thread_slots(const Geometry& g, int tid, int& c, int& hs, int& ps) {
  c = tid & ((1 << g.log2_l) - 1);
  const int slot = tid >> g.log2_l;
  if (g.heads_inner) {
    hs = slot & ((1 << g.log2_hs) - 1);
    ps = slot >> g.log2_hs;
  } else {
    ps = slot & ((1 << g.log2_ps) - 1);
    hs = slot >> g.log2_ps;
  }
}


// Fixed-order sum of column `col` of a [G, C] FP32 array over the rows first,
// first + step, ... (< G): ((0 + p[r0]) + p[r1]) + ... The loads of eight rows
// are issued before their additions, so their latencies overlap, while the
// additions keep the order (and the bits) of the one-row-at-a-time loop.
__device__ __forceinline__ float strided_column_sum(const float* __restrict__ p, int64_t G, int C,
                                                    int col, int first, int step) {
  float v = 0.f;
  int64_t g = first;
  for (; g + 7 * (int64_t)step < G; g += 8 * (int64_t)step) {
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = p[(g + (int64_t)u * step) * C + col];
#pragma unroll
    for (int u = 0; u < 8; ++u) v = __fadd_rn(v, x[u]);
  }
  for (; g < G; g += step) v = __fadd_rn(v, p[g * C + col]);
  return v;
}

}  // namespace flash_prologue
