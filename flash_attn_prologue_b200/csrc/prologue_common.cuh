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

template <typename T, bool VEC>
__device__ __forceinline__ void store_stream(T* p, const Chunk<T>& c) {
  if constexpr (VEC) {
    uint4* p4 = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < Chunk<T>::kWords / 4; ++i)
      __stcs(p4 + i, make_uint4(c.w[4 * i + 0], c.w[4 * i + 1], c.w[4 * i + 2], c.w[4 * i + 3]));
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

// item -> (tensor, b, position block, head group); tensor fastest, then positions.
__device__ __forceinline__ void item_coords(const Geometry& g, int64_t item, int& t, int64_t& b,
                                            int64_t& pb, int64_t& hg) {
  t = (int)(item & 1);
  item >>= 1;
  pb = item % g.n_pos_blocks;
  const int64_t rest = item / g.n_pos_blocks;
  hg = rest % g.n_head_groups;
  b = rest / g.n_head_groups;
}

}  // namespace flash_prologue
