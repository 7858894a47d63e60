// Backward GEMMs of the QKV projection P = X * W^T (sm_100a, tcgen05/TMEM).
//
//   dX[b, n, :]             = sum_{s, h, d} grad_s[b, h, n, d] * W[(s*H + h)*D + d, :]
//   dW[(s*H + h)*D + d, :]  = sum_{b, n}    grad_s[b, h, n, d] * X[b, n, :]
//
// with s = q, k, v. The three gradients are read in their own [B, H, N, D]
// layout (any strides with d contiguous) by 4-D TMA boxes, so dP is never
// gathered; the same views describe a packed [B, N, 3, H, D] dP. This is the
// role of the reference's hand-written backward kernels
// (flash_attn_prologue/gemm_bwd.py:1171-1566: mma.sync on sm_120a, split-K
// partials in BF16).
//
// Both GEMMs use the CTA-pair mainloop of the forward GEMM (qkv_gemm.cu):
// 2-CTA clusters, 256 x 256 output tiles, 128 rows per CTA; per CTA warp 4
// loads its operand halves (two 64 x 64 boxes each for A and B) into a
// 6-stage ring of 32 KB stages whose bytes count on the even CTA's barrier;
// one thread of the even CTA issues tcgen05.mma.cta_group::2 (M = 256,
// N = 256, K = 16); warps 0-3 drain the double-buffered TMEM accumulator
// through 128-byte swizzled staging tiles and TMA stores. Each operand half
// of a 128-deep reduction stage is one TMA box of two 64-column blocks laid
// out block after block (16 KB apart): the gradients are viewed as
// {64, N, D/64, H, B}, so a box {64, 128 tokens, 2, 1, 1} holds whole rows of
// a D = 128 head (or, {64, 128, 1, 2, 1}, of two D = 64 heads), read as full
// 256-byte rows; W as {64, 3HD, hidden/64} and X as {64, N, hidden/64, B}.
//   dX: A (tokens x reduction) is K-major: the two blocks are two 64-deep
//       K blocks; B = W (reduction rows x 128 hidden) is MN-major.
//   dW: A (3HD rows x tokens) and B (hidden x tokens) are both MN-major, the
//       two blocks two 64-wide MN blocks (the descriptors' LBO = 16 KB).
//       When the output tiles alone would leave clusters idle, the
//       token reduction is cut into `split` chunks; each chunk writes FP32
//       partials and a second kernel adds them in chunk order (and casts, or
//       adds the existing dW), so the result does not depend on the schedule.
// No load uses cluster multicast. Every wait is bounded (tma_util.cuh); tensor
// memory is released on every path.
#include <cuda.h>

#include "../../include/flash_prologue.h"
#include "prologue_host.h"
#include "tensor_map.h"
#include "umma_util.cuh"

namespace flash_prologue {
namespace {

constexpr int kBN = 256, kBK = 128;               // reduction block per stage
constexpr int kStages = 3;
constexpr int kBlock = 128 * 64 * 2;               // 128 rows x 64 BF16 (one 128-byte-swizzled block)
constexpr int kStageA = 2 * kBlock;                // 128 rows x 128 of the reduction per CTA
constexpr int kStageBytes = kStageA + 2 * kBlock;  // + B: 128 x 128 per CTA
constexpr int kEpiWarps = 4, kProducerWarp = 4, kMmaWarp = 5;
constexpr int kGemmThreads = 6 * 32;
constexpr int kStageTile = 32 * 128;               // staging tile: 32 rows x 128 B
constexpr int kStagingPerWarp = 2 * kStageTile;
constexpr int kAccCols = kBN, kTmemCols = 2 * kAccCols;
constexpr int kMaxSplit = 8;

enum { kModeDx = 0, kModeDw = 1 };

struct BwdGemmArgs {
  int split;                 // dW: chunks of the token reduction (1 for dX)
  int64_t B, N, H, D, hidden;
  int64_t tiles_n;           // output tiles along hidden (N fastest)
  int64_t tiles;             // all output tiles
  int64_t units;             // tiles * split
  int64_t n_kb;              // 128-deep blocks of the whole reduction
  int64_t m_tiles_per_batch; // dX: ceil(N / 256)
  int64_t kb_per_batch;      // dW: ceil(N / 128)
};

struct BwdMaps {
  CUtensorMap grad[3];  // q, k, v gradients: 5-D {64, N, D/64, H, B}, box {64, 128, 2, 1, 1} (D = 128)
                        // or {64, 128, 1, 2, 1} (D = 64)
  CUtensorMap bop;      // dX: W 3-D {64, 3HD, hidden/64} box {64, 128, 2};
                        // dW: X 4-D {64, N, hidden/64, B} box {64, 128, 2, 1}
  CUtensorMap out;      // dX: {hidden, N, B} BF16 box {64, 32, 1}; dW: {hidden, split*3HD} FP32 box {32, 32}
};

struct BwdSmem {
  unsigned char* ring;
  unsigned char* staging;  // [4 warps][2][kStageTile]
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;      // [2]
  uint64_t* acc_empty;     // [2]
  uint32_t* tmem_slot;
  uint64_t* drain;         // failure path: completion of every MMA issued
};

__device__ __forceinline__ BwdSmem carve(unsigned char* raw) {
  BwdSmem s;
  s.ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  s.staging = s.ring + kStages * kStageBytes;
  s.full = reinterpret_cast<uint64_t*>(s.staging + kEpiWarps * kStagingPerWarp);
  s.empty = s.full + kStages;
  s.acc_full = s.empty + kStages;
  s.acc_empty = s.acc_full + 2;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.acc_empty + 2);
  s.drain = s.acc_empty + 3;  // after the TMEM address slot (16 bytes reserved per 256-byte tail)
  return s;
}
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + kEpiWarps * kStagingPerWarp + 256;

// Output tile, reduction range and chunk of a work unit (chunk-major, then
// tiles with the hidden tile fastest, so clusters working at the same time
// share their A rows and reduction range through L2). Units of odd rounds
// (u / n_pairs odd: the cluster's every second unit) walk the reduction
// backwards, so a round starts on the operand blocks the previous round
// read last, which are still in L2. The direction is fixed by u and the
// grid, so results do not change run to run.
struct Unit {
  int64_t tm, tn, kb_lo, kb_hi;
  int chunk;
  bool reverse;  // walk the reduction from kb_hi - 1 down to kb_lo
};
// Unit and row indices in 32-bit arithmetic: units, tiles, reduction blocks
// and 3HD rows stay below 2^31 (checked on the host), and a 64-bit division is
// a long software sequence.
__device__ __forceinline__ Unit unit_of(const BwdGemmArgs& a, int64_t u, int64_t n_pairs) {
  Unit r;
  const uint32_t u32 = (uint32_t)u, tiles = (uint32_t)a.tiles, tiles_n = (uint32_t)a.tiles_n;
  const uint32_t chunk = u32 / tiles, tile = u32 - chunk * tiles;
  r.chunk = (int)chunk;
  r.tm = tile / tiles_n;
  r.tn = tile - (uint32_t)r.tm * tiles_n;
  r.kb_lo = a.n_kb * r.chunk / a.split;
  r.kb_hi = a.n_kb * (r.chunk + 1) / a.split;
  r.reverse = ((u32 / (uint32_t)n_pairs) & 1) != 0;
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

// (slot, head, first d) of row r of the [3HD] projection axis.
__device__ __forceinline__ void split_row(const BwdGemmArgs& a, int64_t r, int& s, int32_t& h, int32_t& d) {
  const uint32_t hd = (uint32_t)(a.H * a.D), r32 = (uint32_t)r, dd = (uint32_t)a.D;
  s = (int)(r32 / hd);
  const uint32_t rem = r32 - (uint32_t)s * hd;
  h = (int32_t)(rem / dd);
  d = (int32_t)(rem - (uint32_t)h * dd);
}

}  // namespace

// ---------------------------------------------------------------------------
// The kernel: MODE kModeDx or kModeDw (see the file comment).
template <int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    qkv_bwd_gemm_kernel(const __grid_constant__ BwdMaps maps, const __grid_constant__ BwdGemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  const BwdSmem sm = carve(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the CTA that issues the MMAs
  const int64_t pair = blockIdx.x >> 1;
  const int64_t n_pairs = gridDim.x >> 1;
  constexpr uint32_t kBar = sizeof(uint64_t);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);   // even CTA: its producer's arrival + both CTAs' bytes
      mbar_init(&sm.empty[s], 1);  // one MMA commit per use, in each CTA
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 2 * kEpiWarps);  // even CTA: the epilogue warps of both CTAs
    }
    mbar_init(sm.drain, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(sm.tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *sm.tmem_slot;

  if (warp == kProducerWarp) {
    // -------------------- TMA producer (both CTAs) --------------------
    if (lane == 0) {
      for (int i = 0; i < 3; ++i) prefetch_tmap(&maps.grad[i]);
      prefetch_tmap(&maps.bop);
      const uint32_t full0 = mapa_shared(smem_u32(sm.full), 0);
      // dX: every cluster reads all of W (25 MB at C5) again for each of its
      // tiles; kept in L2 ahead of the streamed gradients.
      const uint64_t pol_w = policy_evict_last();
      bool failed = false;
      uint32_t it = 0;
      for (int64_t u = pair; u < a.units && !failed; u += n_pairs) {
        const Unit un = unit_of(a, u, n_pairs);
        const int32_t col0 = (int32_t)(un.tn * kBN + rank * 128);  // hidden column of B
        // dX: this CTA's 128 tokens; dW: this CTA's 128 rows of 3HD (two boxes).
        int32_t b_x = 0, n0 = 0;
        int s0 = 0;
        int32_t h0 = 0, d0 = 0;
        if (MODE == kModeDx) {
          b_x = (int32_t)(un.tm / a.m_tiles_per_batch);
          n0 = (int32_t)((un.tm % a.m_tiles_per_batch) * kBN + rank * 128);
        } else {
          // 128 rows starting at a multiple of 128: within one slot (H*D is a
          // multiple of 256), one D = 128 head or two D = 64 heads.
          split_row(a, un.tm * kBN + rank * 128, s0, h0, d0);
        }
        for (int64_t j = 0; j < un.kb_hi - un.kb_lo; ++j, ++it) {
          const int64_t kb = un.reverse ? un.kb_hi - 1 - j : un.kb_lo + j;
          const int s = it % kStages;
          if (!mbar_wait(&sm.empty[s], ((it / kStages) & 1) ^ 1)) { failed = true; break; }
          unsigned char* st = sm.ring + s * kStageBytes;
          const uint32_t bar = full0 + s * kBar;
          if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], 2 * kStageBytes);
          if (MODE == kModeDx) {
            // Reduction rows kb*128 .. +127: one D = 128 head or two D = 64 heads.
            int slot;
            int32_t h, d;
            split_row(a, kb * kBK, slot, h, d);
            tma_load_5d_pair(st, &maps.grad[slot], 0, n0, d / 64, h, b_x, bar);
            tma_load_3d_pair_hint(st + kStageA, &maps.bop, 0, (int32_t)(kb * kBK), col0 / 64, bar, pol_w);
          } else {
            const int32_t bb = (int32_t)(kb / a.kb_per_batch);
            const int32_t t0 = (int32_t)((kb % a.kb_per_batch) * kBK);
            tma_load_5d_pair(st, &maps.grad[s0], 0, t0, d0 / 64, h0, bb, bar);
            tma_load_4d_pair(st + kStageA, &maps.bop, 0, t0, col0 / 64, bb, bar);
          }
        }
      }
      // Drain: the MMA commits of the last uses of every stage must have
      // arrived on this CTA's empty barriers before the CTA may end.
      for (int j = 0; j < kStages && !failed; ++j, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&sm.empty[s], ((it / kStages) & 1) ^ 1)) failed = true;
      }
    }
  } else if (warp == kMmaWarp) {
    // -------------------- MMA issuer (even CTA, one thread) --------------------
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32_major(2 * 128, kBN, MODE == kModeDw, true);
      const uint32_t empty_own = mapa_shared(smem_u32(sm.empty), 0);
      const uint32_t empty_peer = mapa_shared(smem_u32(sm.empty), 1);
      const uint32_t accf_own = mapa_shared(smem_u32(sm.acc_full), 0);
      const uint32_t accf_peer = mapa_shared(smem_u32(sm.acc_full), 1);
      bool failed = false;
      uint32_t it = 0, tcount = 0;
      for (int64_t u = pair; u < a.units && !failed; u += n_pairs, ++tcount) {
        const Unit un = unit_of(a, u, n_pairs);
        const uint32_t abuf = tcount & 1;
        if (!mbar_wait_cluster(&sm.acc_empty[abuf], ((tcount >> 1) & 1) ^ 1)) { failed = true; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + abuf * kAccCols;
        for (int64_t j = 0; j < un.kb_hi - un.kb_lo; ++j, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&sm.full[s], (it / kStages) & 1)) { failed = true; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(sm.ring + s * kStageBytes);
          const uint32_t sb = sa + kStageA;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major A: two 64-deep blocks, +32 bytes along K per step within
            // one; MN-major operands: +2 swizzle atoms (16 K-rows) per step.
            const uint64_t adesc = (MODE == kModeDx)
                                       ? smem_desc_k_sw128(sa + (kk >> 2) * kBlock) + 2 * (kk & 3)
                                       : smem_desc_mn_sw128(sa + kk * 2048, kBlock);
            const uint64_t bdesc = smem_desc_mn_sw128(sb + kk * 2048, kBlock);
            umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (j != 0 || kk != 0) ? 1u : 0u);
          }
          umma_commit_pair(empty_own + s * kBar);
          umma_commit_pair(empty_peer + s * kBar);
        }
        if (failed) break;
        umma_commit_pair(accf_own + abuf * kBar);
        umma_commit_pair(accf_peer + abuf * kBar);
      }
      // Wait for the last accumulator's MMAs before TMEM may be released.
      if (tcount > 0 && !failed) {
        const uint32_t last = tcount - 1;
        mbar_wait(&sm.acc_full[last & 1], (last >> 1) & 1);
      }
      // A timed-out wait skipped that: wait (bounded) for every MMA issued so
      // far through one more commit, so TMEM is not released under them.
      if (failed && it > 0) {
        umma_commit_pair(mapa_shared(smem_u32(sm.drain), 0));
        mbar_wait(sm.drain, 0);
      }
    }
  } else {
    // -------------------- epilogue (warps 0-3, both CTAs) --------------------
    // Warp w drains TMEM lanes 32w .. 32w + 31 (its 32 output rows) through two
    // staging tiles of 32 rows x 128 bytes (128-byte swizzle), one TMA store each.
    unsigned char* const stage_base = sm.staging + warp * kStagingPerWarp;
    int cur = 0;
    const uint32_t acc_empty0 = mapa_shared(smem_u32(sm.acc_empty), 0);
    auto stage_next = [&]() -> unsigned char* {
      if (lane == 0) bulk_wait_group_read<1>();  // the store issued from this buffer has read it
      __syncwarp();
      unsigned char* t = stage_base + cur * kStageTile;
      cur ^= 1;
      return t;
    };
    auto put16 = [&](unsigned char* tile, int chunk, uint4 v) {
      *reinterpret_cast<uint4*>(tile + lane * 128 + ((chunk ^ (lane & 7)) << 4)) = v;
    };
    uint32_t tcount = 0;
    for (int64_t u = pair; u < a.units; u += n_pairs, ++tcount) {
      const Unit un = unit_of(a, u, n_pairs);
      const uint32_t abuf = tcount & 1;
      if (!mbar_wait(&sm.acc_full[abuf], (tcount >> 1) & 1)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + abuf * kAccCols + ((uint32_t)(warp * 32) << 16);
      const int32_t col0 = (int32_t)(un.tn * kBN);  // each CTA's accumulator holds all 256 columns
      if (MODE == kModeDx) {
        const int32_t bb = (int32_t)(un.tm / a.m_tiles_per_batch);
        const int32_t row0 = (int32_t)((un.tm % a.m_tiles_per_batch) * kBN + rank * 128 + warp * 32);
#pragma unroll 1
        for (int c = 0; c < kBN / 64; ++c) {  // 64 BF16 columns per staging tile
          uint32_t v[32], w[32];
          tmem_ld32(tbase + 64 * c, v);
          tmem_ld32(tbase + 64 * c + 32, w);
          tmem_wait_ld();
          unsigned char* tile = stage_next();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              p[i] = pack_bf16x2(__uint_as_float(v[8 * q + 2 * i]), __uint_as_float(v[8 * q + 2 * i + 1]));
            put16(tile, q, make_uint4(p[0], p[1], p[2], p[3]));
#pragma unroll
            for (int i = 0; i < 4; ++i)
              p[i] = pack_bf16x2(__uint_as_float(w[8 * q + 2 * i]), __uint_as_float(w[8 * q + 2 * i + 1]));
            put16(tile, 4 + q, make_uint4(p[0], p[1], p[2], p[3]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&maps.out, col0 + 64 * c, row0, bb, tile);
            bulk_commit_group();
          }
        }
      } else {
        const int32_t row0 = (int32_t)(un.chunk * 3 * a.H * a.D + un.tm * kBN + rank * 128 + warp * 32);
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {  // 32 FP32 columns per staging tile
          uint32_t v[32];
          tmem_ld32(tbase + 32 * c, v);
          tmem_wait_ld();
          unsigned char* tile = stage_next();
#pragma unroll
          for (int q = 0; q < 8; ++q) put16(tile, q, make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&maps.out, col0 + 32 * c, row0, tile);
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + abuf * kBar);
    }
    // Every store must have completed before the CTA ends.
    if (lane == 0) bulk_wait_group0();
  }

  // Teardown: every thread of both CTAs arrives here (also after a timed-out
  // wait), so no CTA ends while its peer may still signal its barriers.
  tc_fence_before();
  __syncwarp();
  cluster_sync();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// dW from the split partials: dW[i] = BF16(((p_0[i] + p_1[i]) + ...) [+ dW[i]]),
// four elements per thread and step, in chunk order.
__global__ void __launch_bounds__(256)
    qkv_bwd_dw_finalize_kernel(const float* __restrict__ part, int split, int64_t count,
                               __nv_bfloat16* __restrict__ dw, int accumulate) {
  const int64_t n4 = count / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = reinterpret_cast<const float4*>(part)[i];
    for (int j = 1; j < split; ++j) {
      const float4 v = reinterpret_cast<const float4*>(part + (int64_t)j * count)[i];
      s.x = __fadd_rn(s.x, v.x);
      s.y = __fadd_rn(s.y, v.y);
      s.z = __fadd_rn(s.z, v.z);
      s.w = __fadd_rn(s.w, v.w);
    }
    uint2* out = reinterpret_cast<uint2*>(dw) + i;
    if (accumulate) {
      const uint2 o = *out;
      s.x = __fadd_rn(s.x, __uint_as_float(o.x << 16));
      s.y = __fadd_rn(s.y, __uint_as_float(o.x & 0xFFFF0000u));
      s.z = __fadd_rn(s.z, __uint_as_float(o.y << 16));
      s.w = __fadd_rn(s.w, __uint_as_float(o.y & 0xFFFF0000u));
    }
    *out = make_uint2(pack_bf16x2(s.x, s.y), pack_bf16x2(s.z, s.w));
  }
}

// ---------------------------------------------------------------------------
// Host side

namespace {

int device_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return sms;
}

// Launch configuration of the MODE kernel on `sms` SMs and the number of its
// 2-CTA clusters that can be resident at once (cached per device; 0 if none).
template <int MODE>
int bwd_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, cudaStream_t stream) {
  static int cached[64] = {0};
  const void* fn = reinterpret_cast<const void*>(&qkv_bwd_gemm_kernel<MODE>);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
    return 0;
  const int sms = device_sms();
  if (sms < 2) return 0;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3((unsigned)(sms & ~1));
  cfg->blockDim = dim3(kGemmThreads);
  cfg->dynamicSmemBytes = kSmemBytes;
  cfg->stream = stream;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, qkv_bwd_gemm_kernel<MODE>, cfg) != cudaSuccess) return 0;
  if (dev < 64) cached[dev] = n;
  return n;
}

// Chunks of the dW token reduction: the smallest count whose units fill the
// clusters' last wave clearly better (each chunk keeps >= 4 blocks of 64 tokens).
int dw_split(int64_t tiles, int64_t n_kb, int pairs) {
  if (pairs <= 0) return 1;
  auto eff = [&](int s) {
    const int64_t units = tiles * s;
    const int64_t waves = (units + pairs - 1) / pairs;
    return (double)units / (double)(waves * pairs);
  };
  int best = 1;
  double best_eff = eff(1);
  for (int s = 2; s <= kMaxSplit && n_kb >= 4 * (int64_t)s; ++s) {
    const double e = eff(s);
    if (e > best_eff + 0.03) {
      best = s;
      best_eff = e;
    }
  }
  return best;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Map of one [B, H, N, D] gradient view (element strides st[0..3] = b, h, n,
// d; d must be 1) as 5-D {64, N, D/64, H, B}, 128-byte swizzle, box {64, 128
// tokens} x two 64-row blocks: the d blocks of a D = 128 head, or two D = 64
// heads, laid out block after block. Dimensions of extent 1 get a
// placeholder stride (never used for addressing).
bool grad_map(CUtensorMap* m, const void* base, const int64_t st[4], int64_t B, int64_t H, int64_t N,
              int64_t D) {
  if (!base || !al16(base) || st[3] != 1) return false;
  int64_t sb = st[0], sh = st[1], sn = st[2];
  if (N == 1) sn = D;
  if (H == 1) sh = D;
  if (B == 1) sb = D;
  if (sn <= 0 || sh <= 0 || sb <= 0 || (sn | sh | sb) % 8 != 0) return false;
  const uint64_t dims[5] = {64, (uint64_t)N, (uint64_t)(D / 64), (uint64_t)H, (uint64_t)B};
  const uint64_t strides[4] = {(uint64_t)sn * 2, 128, (uint64_t)sh * 2, (uint64_t)sb * 2};
  const uint32_t box[5] = {64, 128, D == 128 ? 2u : 1u, D == 128 ? 1u : 2u, 1};
  return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, base, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

// [B, N, hidden] contiguous BF16 as a 3-D map {hidden, N, B} with box {64, rows, 1}.
bool bnh_map(CUtensorMap* m, const void* base, int64_t B, int64_t N, int64_t hidden, uint32_t rows) {
  if (!base || !al16(base)) return false;
  const uint64_t dims[3] = {(uint64_t)hidden, (uint64_t)N, (uint64_t)B};
  const uint64_t strides[2] = {(uint64_t)hidden * 2, (uint64_t)(N * hidden) * 2};
  const uint32_t box[3] = {64, rows, 1};
  return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

// An MN-major B operand: the row-major [rows, hidden] matrix (rows = the
// reduction index) viewed as {64, rows, hidden/64 blocks[, B]} so one box
// {64, 128 rows, 2 blocks[, 1]} brings 128 hidden columns, block after block.
// dX: W with rows = 3HD (3-D); dW: x [B, N, hidden] with rows = N (4-D).
bool mn_b_map(CUtensorMap* m, const void* base, int64_t rows, int64_t hidden, int64_t B, bool batched) {
  if (!base || !al16(base)) return false;
  const uint64_t dims[4] = {64, (uint64_t)rows, (uint64_t)(hidden / 64), (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)hidden * 2, 128, (uint64_t)(rows * hidden) * 2};
  const uint32_t box[4] = {64, 128, 2, 1};
  return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, batched ? 4 : 3, base, dims, strides,
                           box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int check_common(int64_t B, int64_t H, int64_t N, int64_t D, int64_t hidden) {
  if (B < 0 || H <= 0 || N < 0 || hidden < 0) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (D != 64 && D != 128) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if ((H * D) % kBN != 0 || hidden % 64 != 0) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (N >= (int64_t(1) << 31) || B >= (int64_t(1) << 31) || 3 * H * D * kMaxSplit >= (int64_t(1) << 31) ||
      hidden >= (int64_t(1) << 31))
    return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  return FLASH_PROLOGUE_OK;
}

bool make_grad_maps(BwdMaps* maps, const void* gq, const int64_t* sq, const void* gk, const int64_t* sk,
                    const void* gv, const int64_t* sv, int64_t B, int64_t H, int64_t N, int64_t D) {
  return grad_map(&maps->grad[0], gq, sq, B, H, N, D) && grad_map(&maps->grad[1], gk, sk, B, H, N, D) &&
         grad_map(&maps->grad[2], gv, sv, B, H, N, D);
}

template <int MODE>
cudaError_t launch_bwd_gemm(const BwdMaps& maps, BwdGemmArgs& a, int pairs_max, cudaStream_t stream) {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  if (bwd_config<MODE>(&cfg, attr, stream) <= 0 || pairs_max <= 0) return cudaErrorInvalidConfiguration;
  const int64_t pairs = a.units < pairs_max ? a.units : pairs_max;
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  return cudaLaunchKernelEx(&cfg, qkv_bwd_gemm_kernel<MODE>, maps, a);
}

// The dW plan: args (tiles, split, ...) and the workspace it needs.
int dw_plan(int64_t B, int64_t H, int64_t N, int64_t D, int64_t hidden, cudaStream_t stream,
            BwdGemmArgs* a, int* pairs_out) {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  const int pairs = bwd_config<kModeDw>(&cfg, attr, stream);
  if (pairs <= 0) return FLASH_PROLOGUE_ERR_CUDA;
  *a = BwdGemmArgs{};
  a->B = B; a->N = N; a->H = H; a->D = D; a->hidden = hidden;
  a->tiles_n = (hidden + kBN - 1) / kBN;
  a->tiles = (3 * H * D / kBN) * a->tiles_n;
  a->kb_per_batch = (N + kBK - 1) / kBK;
  a->n_kb = B * a->kb_per_batch;
  a->split = dw_split(a->tiles, a->n_kb, pairs);
  a->units = a->tiles * a->split;
  *pairs_out = pairs;
  return FLASH_PROLOGUE_OK;
}

}  // namespace

// The error word of this translation unit's bounded waits (tma_util.cuh).
cudaError_t read_gemm_bwd_device_error(int* value, bool reset) {
  cudaError_t err = cudaMemcpyFromSymbol(value, g_device_error, sizeof(int));
  if (err != cudaSuccess || !reset) return err;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
}

}  // namespace flash_prologue

using namespace flash_prologue;

extern "C" {

FLASH_PROLOGUE_API int flash_prologue_qkv_bwd_dx(
    const void* grad_q, const int64_t gq_strides[4], const void* grad_k, const int64_t gk_strides[4],
    const void* grad_v, const int64_t gv_strides[4], const void* weight, void* grad_x, int64_t B,
    int64_t H, int64_t N, int64_t D, int64_t hidden, void* stream) {
  int rc = check_common(B, H, N, D, hidden);
  if (rc != FLASH_PROLOGUE_OK) return rc;
  if (B * N == 0 || hidden == 0) return FLASH_PROLOGUE_OK;
  if (!gq_strides || !gk_strides || !gv_strides || !weight || !grad_x)
    return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (!al16(weight) || !al16(grad_x)) return FLASH_PROLOGUE_ERR_ALIGNMENT;
  BwdMaps maps;
  if (!make_grad_maps(&maps, grad_q, gq_strides, grad_k, gk_strides, grad_v, gv_strides, B,
                      H, N, D))
    return FLASH_PROLOGUE_ERR_ALIGNMENT;
  if (!mn_b_map(&maps.bop, weight, 3 * H * D, hidden, 1, false) ||
      !bnh_map(&maps.out, grad_x, B, N, hidden, 32))
    return FLASH_PROLOGUE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  const int pairs = bwd_config<kModeDx>(&cfg, attr, s);
  if (pairs <= 0) return FLASH_PROLOGUE_ERR_CUDA;
  BwdGemmArgs a{};
  a.split = 1;
  a.B = B; a.N = N; a.H = H; a.D = D; a.hidden = hidden;
  a.m_tiles_per_batch = (N + kBN - 1) / kBN;
  a.tiles_n = (hidden + kBN - 1) / kBN;
  a.tiles = B * a.m_tiles_per_batch * a.tiles_n;
  a.units = a.tiles;
  a.n_kb = 3 * H * D / kBK;
  return launch_bwd_gemm<kModeDx>(maps, a, pairs, s) == cudaSuccess ? FLASH_PROLOGUE_OK
                                                                     : FLASH_PROLOGUE_ERR_CUDA;
}

FLASH_PROLOGUE_API int flash_prologue_qkv_bwd_dw_workspace_size(int64_t B, int64_t H, int64_t N,
                                                                 int64_t D, int64_t hidden,
                                                                 size_t* bytes) {
  if (!bytes) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  *bytes = 0;
  const int rc = check_common(B, H, N, D, hidden);
  if (rc != FLASH_PROLOGUE_OK) return rc;
  if (B * N == 0 || hidden == 0) return FLASH_PROLOGUE_OK;
  BwdGemmArgs a;
  int pairs = 0;
  const int prc = dw_plan(B, H, N, D, hidden, nullptr, &a, &pairs);
  if (prc != FLASH_PROLOGUE_OK) return prc;
  *bytes = (size_t)a.split * (size_t)(3 * H * D * hidden) * sizeof(float);
  return FLASH_PROLOGUE_OK;
}

FLASH_PROLOGUE_API int flash_prologue_qkv_bwd_dw(
    const void* grad_q, const int64_t gq_strides[4], const void* grad_k, const int64_t gk_strides[4],
    const void* grad_v, const int64_t gv_strides[4], const void* x, void* grad_w, int accumulate,
    void* workspace, size_t workspace_bytes, int64_t B, int64_t H, int64_t N, int64_t D,
    int64_t hidden, void* stream) {
  int rc = check_common(B, H, N, D, hidden);
  if (rc != FLASH_PROLOGUE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (hidden == 0) return FLASH_PROLOGUE_OK;
  if (!grad_w) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (!al16(grad_w)) return FLASH_PROLOGUE_ERR_ALIGNMENT;
  const int64_t count = 3 * H * D * hidden;
  if (B * N == 0) {  // an empty sum: zeros, or the accumulator unchanged
    if (accumulate) return FLASH_PROLOGUE_OK;
    return cudaMemsetAsync(grad_w, 0, (size_t)count * 2, s) == cudaSuccess ? FLASH_PROLOGUE_OK
                                                                           : FLASH_PROLOGUE_ERR_CUDA;
  }
  if (!gq_strides || !gk_strides || !gv_strides || !x || !workspace)
    return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (!al16(x) || !al16(workspace)) return FLASH_PROLOGUE_ERR_ALIGNMENT;
  BwdGemmArgs a;
  int pairs = 0;
  rc = dw_plan(B, H, N, D, hidden, s, &a, &pairs);
  if (rc != FLASH_PROLOGUE_OK) return rc;
  if (workspace_bytes < (size_t)a.split * (size_t)count * sizeof(float))
    return FLASH_PROLOGUE_ERR_WORKSPACE;
  BwdMaps maps;
  if (!make_grad_maps(&maps, grad_q, gq_strides, grad_k, gk_strides, grad_v, gv_strides, B,
                      H, N, D))
    return FLASH_PROLOGUE_ERR_ALIGNMENT;
  const uint64_t odims[2] = {(uint64_t)hidden, (uint64_t)(a.split * 3 * H * D)};
  const uint64_t ostr[1] = {(uint64_t)hidden * 4};
  const uint32_t obox[2] = {32, 32};
  if (!mn_b_map(&maps.bop, x, N, hidden, B, true) ||
      !encode_tensor_map(&maps.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, workspace, odims, ostr, obox,
                         CU_TENSOR_MAP_SWIZZLE_128B))
    return FLASH_PROLOGUE_ERR_CUDA;
  if (launch_bwd_gemm<kModeDw>(maps, a, pairs, s) != cudaSuccess) return FLASH_PROLOGUE_ERR_CUDA;
  const int sms = device_sms();
  const int64_t blocks = (count / 4 + 255) / 256;
  const int grid = (int)(blocks < 4LL * sms ? blocks : 4LL * sms);
  return launch_kernel(qkv_bwd_dw_finalize_kernel, dim3(grid), dim3(256), 0, s,
                       static_cast<const float*>(workspace), a.split, count,
                       static_cast<__nv_bfloat16*>(grad_w), accumulate ? 1 : 0) == cudaSuccess
             ? FLASH_PROLOGUE_OK
             : FLASH_PROLOGUE_ERR_CUDA;
}

}  // extern "C"
