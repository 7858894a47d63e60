// Fused QKV projection GEMM with the prologue in its epilogue (sm_100a).
//
// Computes P = X * W^T for X [M, K] BF16 (tokens x hidden) and W [3*H*D, K]
// BF16 (nn.Linear layout, rows = Q heads | K heads | V heads), rounds P to BF16
// (the projection a BF16 linear layer outputs), and then, per token and head:
// Q, K -> RMSNorm (FP32 weight) -> split-half RoPE (FP32 sin/cos of the
// token's position) -> Q * exp(scale[h]) -> BF16; V is stored as projected.
// Outputs are [B, H, S, D] with M = B * S. Optionally the BF16 Q/K projections
// before the prologue are stored too (what the backward needs). This replaces
// the reference's GEMM launch + two copies + in-place prologue launch
// (flash_attn_prologue/fused_qkv.py:698-825) with one kernel.
//
// Two mainloops share one epilogue:
//
// * CTA pair (default): 2-CTA clusters, one persistent pair per two SMs. A
//   tile is 256 tokens x 256 output columns. Each CTA's warp 4 loads its own
//   halves -- X rows [m0 + 128*rank, +128) and W rows [n0 + 128*rank, +128),
//   64 columns of K per stage, 128-byte swizzled -- into a 5-stage ring; all
//   four loads of a stage count their bytes on the even CTA's full barrier.
//   One thread of the even CTA issues tcgen05.mma.cta_group::2 (M = 256,
//   N = 256, K = 16): the tensor cores of both SMs read A from their own
//   shared memory and B from both, and each CTA's tensor memory receives its
//   128 rows. Per SM this moves 32 KB of operands per 128x256x64 of work
//   instead of 48 KB, which is what limits the single-CTA loop.
// * Single CTA: one persistent CTA per SM, 128 x 256 tiles, 4-stage ring of
//   48 KB stages, tcgen05.mma.cta_group::1 (M = 128).
//
// In both, warp 5 owns the 512 tensor-memory columns (two 256-column FP32
// accumulators, so tile i's epilogue overlaps tile i+1's MMAs) and warps 0-3
// are the epilogue: tcgen05.ld of the accumulator (TMEM lane = token row),
// BF16 rounding, sum of squares over the head, RoPE pairing of columns j and
// j + D/2 (both in the same thread), stores through swizzled staging tiles and
// TMA tensor stores. Tiles are ordered with the N tile fastest, so CTAs working
// at the same time share X rows through L2 (W stays L2-resident). No load uses
// cluster multicast. All waits are bounded (tma_util.cuh); a timeout records
// an error, and tensor memory is released on every path.
#include <cuda.h>

#include "../../include/flash_prologue.h"
#include "prologue_common.cuh"
#include "prologue_host.h"
#include "tensor_map.h"
#include "umma_util.cuh"

namespace flash_prologue {
namespace {

constexpr int BN = 256, BK = 64;
constexpr int kAccCols = BN;                    // FP32 columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;         // two accumulators = all 512 columns
// Warp roles: warps 0 .. EPI-1 epilogue, EPI the TMA producer, EPI+1 the
// TMEM owner / MMA issuer.
template <int EPI>
struct Roles {
  static constexpr int kEpi = EPI;
  static constexpr int kProducer = EPI;
  static constexpr int kMma = EPI + 1;
  static constexpr int kThreads = (EPI + 2) * 32;
};
// Output staging: per epilogue warp, its 32 rows of one head as [32][128 B]
// halves (64 BF16 columns each), 128-byte swizzled, written out by TMA stores.
constexpr int kStageHalfBytes = 32 * 128;
constexpr int kStagingPerWarp = 2 * kStageHalfBytes;  // up to D = 128

// Single-CTA mainloop: 128 x 256 tiles, 4 epilogue warps.
using RolesSingle = Roles<4>;
constexpr int kRowsSingle = 128;
constexpr int kStagesSingle = 4;
constexpr int kStagingBufsSingle = 1;
constexpr int kStageASingle = kRowsSingle * BK * 2;            // 16 KB
constexpr int kStageBytesSingle = kStageASingle + BN * BK * 2;  // 48 KB

// CTA-pair mainloop: 256 x 256 tiles, per CTA 128 rows of X and 128 of W.
// Two configurations: with the prologue, 8 epilogue warps (two per SM
// sub-partition, so one's latency hides under the other's work; 168 registers
// a thread) and 5 stages; plain projection, 4 epilogue warps and 6 stages.
constexpr int kRowsPair = 256;
constexpr int kStagingBufsPair = 1;
template <int EPI>
struct PairConfig {
  using R = Roles<EPI>;
  static constexpr int kStages = EPI == 8 ? 5 : 6;
  static constexpr int kSlots = 1;  // sin/cos ring slots
};
constexpr int kStageAPair = 128 * BK * 2;                         // 16 KB
constexpr int kStageBytesPair = kStageAPair + (BN / 2) * BK * 2;  // 32 KB

struct GemmArgs {
  int64_t M, K, H, D, S;          // S = tokens per batch (M = B * S)
  int64_t n_tiles_n, n_tiles;     // tiles of the mainloop in use (N tile fastest)
  const float* w;                 // RMSNorm weight [2, D]
  const float* scales;            // [H]
  const float* sin;
  const float* cos;
  int64_t sin_b, sin_n, cos_b, cos_n;  // element strides; j stride 1
  void* out[3];                   // q, k, v as [B, H, S, D]
  void* raw[2];                   // optional BF16 q, k projections [B, H, S, D]
  float eps;
  int apply_prologue;
  int tma_store;                  // 1: outputs through per-warp staging + TMA stores (S % 32 == 0)
};

// Tensor maps of the five outputs as 2-D [B*H*S rows, D columns] BF16 tensors
// with a (64 x 32) box and 128-byte swizzle: q, k, v, raw q, raw k.
struct OutMaps {
  CUtensorMap m[5];
};

__device__ __forceinline__ uint32_t pack_bf16(float2 v) {
  __nv_bfloat162 p = __floats2bfloat162_rn(v.x, v.y);
  return *reinterpret_cast<uint32_t*>(&p);
}

// The two BF16 values of a packed pair as FP32 (exact).
__device__ __forceinline__ float2 unpack_bf16(uint32_t p) {
  return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u));
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Shared-memory carve-up common to both kernels: the operand ring (1024-byte
// aligned), then the epilogue staging, barriers, the TMEM address slot and the
// RMSNorm weight. Both CTAs of a pair get the same offsets.
struct GemmSmem {
  unsigned char* ring;
  unsigned char* staging;  // [epilogue warps][NBUF][kStagingPerWarp]
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;      // [2]
  uint64_t* acc_empty;     // [2]
  uint32_t* tmem_slot;
  uint64_t* drain;         // failure path: completion of every MMA issued (see the MMA issuers)
  float* w_s;              // [2 * D]
};

template <int STAGES, int STAGE_BYTES, int NBUF, int EPI>
__device__ __forceinline__ GemmSmem carve_smem(unsigned char* smem_raw) {
  GemmSmem s;
  s.ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                            ~uintptr_t(1023));
  s.staging = s.ring + STAGES * STAGE_BYTES;
  s.full = reinterpret_cast<uint64_t*>(s.staging + EPI * NBUF * kStagingPerWarp);
  s.empty = s.full + STAGES;
  s.acc_full = s.empty + STAGES;
  s.acc_empty = s.acc_full + 2;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.acc_empty + 2);
  s.drain = reinterpret_cast<uint64_t*>(s.tmem_slot + 2);  // 8-byte aligned: acc_empty is
  s.w_s = reinterpret_cast<float*>(s.tmem_slot + 4);
  return s;
}

constexpr size_t smem_bytes_for(int stages, int stage_bytes, int nbuf, int epi, int64_t D) {
  return 1024 + (size_t)stages * stage_bytes + (size_t)epi * nbuf * kStagingPerWarp + 256 +
         (size_t)(2 * D) * 4;
}

}  // namespace

// ---------------------------------------------------------------------------
// Epilogue (warps 0 .. EPI-1). Processes the tiles tile0, tile0 + step, ...;
// this CTA's accumulator rows are tokens (tile / n_tiles_n) * ROWS + m_off +
// row. Warp w reads TMEM lanes 32 * (w % 4) .. + 31 (a warp may only access
// its quarter of the lanes), so with EPI = 8 the warps w and w + 4 share rows
// and split the heads of the tile between them. After reading an accumulator
// each warp arrives once on acc_empty[buffer]: this CTA's barrier, or for a
// pair the even CTA's, at the shared::cluster address acc_empty_cluster
// (+ 8 bytes per buffer).
template <int D, int ROWS, int NBUF, int EPI, int SLOTS>
__device__ __forceinline__ void run_epilogue(const OutMaps& om, const GemmArgs& a, const GemmSmem& sm,
                                             uint32_t tmem_base, int64_t tile0, int64_t step,
                                             int m_off, uint32_t acc_empty_cluster) {
  constexpr int HALF = D / 2;
  constexpr int HEADS_PER_TILE = BN / D;
  constexpr int GROUPS = HALF / 16;     // 16-column groups of each half of a head
  constexpr int HEAD_STEP = EPI / 4;    // warps sharing a lane quarter split the heads
  static_assert(HEADS_PER_TILE % HEAD_STEP == 0, "heads per warp");
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quarter = warp & 3;
  const int head0 = warp >> 2;
  const int row = quarter * 32 + lane;  // TMEM lane == accumulator row
  unsigned char* const stage_base = sm.staging + warp * NBUF * kStagingPerWarp;
  unsigned char* stage_w = stage_base;  // the staging tile being filled
  int cur = 0;
  const bool staged = a.tma_store != 0;
  // 16 output bytes (8 BF16 at column `col` of the head) of this thread's row:
  // into the warp's swizzled staging tile, or straight to global memory.
  auto emit16 = [&](__nv_bfloat16* grow, bool valid, int col, uint4 v) {
    if (staged) {
      unsigned char* half = stage_w + (col >> 6) * kStageHalfBytes;
      const int chunk = (col & 63) >> 3;
      *reinterpret_cast<uint4*>(half + lane * 128 + ((chunk ^ (lane & 7)) << 4)) = v;
    } else if (valid) {
      *reinterpret_cast<uint4*>(grow + col) = v;
    }
  };
  // Staged path: write the warp's 32 rows of one head to `map` at row0 (one
  // bulk group) and move on to the next staging tile ...
  auto flush = [&](const CUtensorMap* map, int64_t row0) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      for (int half = 0; half < D / 64; ++half)
        tma_store_2d(map, half * 64, (int32_t)row0, stage_w + half * kStageHalfBytes);
      bulk_commit_group();
    }
    cur = (cur + 1 == NBUF) ? 0 : cur + 1;
    stage_w = stage_base + cur * kStagingPerWarp;
  };
  // ... and before filling a staging tile, wait until the stores issued from
  // it (NBUF groups ago) have read it.
  auto reclaim = [&]() {
    if (lane == 0) bulk_wait_group_read<NBUF - 1>();
    __syncwarp();
  };
  // The token's sin/cos values, 16 of each per group, in a ring of SLOTS group
  // slots: the first SLOTS groups are requested before the accumulator wait
  // (and again at the start of each further head when a head has more groups
  // than slots), group g + SLOTS as soon as group g has been used.
  static_assert(SLOTS >= 1 && SLOTS <= GROUPS, "sin/cos ring");
  float sn[SLOTS][16], cs[SLOTS][16];
  const float* srow = a.sin;
  const float* crow = a.cos;
  bool valid = false;
  auto load_group = [&](int g, int slot) {
    if (valid) {
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 s4 = ldg4(srow + 16 * g + j), c4 = ldg4(crow + 16 * g + j);
        sn[slot][j] = s4.x; sn[slot][j + 1] = s4.y; sn[slot][j + 2] = s4.z; sn[slot][j + 3] = s4.w;
        cs[slot][j] = c4.x; cs[slot][j + 1] = c4.y; cs[slot][j + 2] = c4.z; cs[slot][j + 3] = c4.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) { sn[slot][j] = 0.f; cs[slot][j] = 0.f; }
    }
  };
  // Tile and token indices in 32-bit arithmetic (the host checks that tiles,
  // tokens and M * H stay below 2^31): a 64-bit division is a long software
  // sequence, and this runs once per tile in every epilogue thread.
  const uint32_t n_tn = (uint32_t)a.n_tiles_n;
  const uint32_t s32 = (uint32_t)a.S;
  const uint32_t tiles_per_seg = (uint32_t)(a.H * D / BN);  // H * D is a multiple of BN
  uint32_t tcount = 0;
  for (int64_t tile = tile0; tile < a.n_tiles; tile += step, ++tcount) {
    const uint32_t abuf = tcount & 1;
    const uint32_t tm = (uint32_t)tile / n_tn, tn = (uint32_t)tile - tm * n_tn;
    const uint32_t mrow0 = tm * ROWS + (uint32_t)m_off;
    const uint32_t m = mrow0 + row;
    valid = (int64_t)m < a.M;
    const uint32_t b32 = m / s32;
    const int64_t b = b32, sp = m - b32 * s32;
    // First token of this warp's 32 rows (S % 32 == 0 on the staged path,
    // so all 32 share its batch index).
    const uint32_t mw = mrow0 + quarter * 32;
    const uint32_t bw32 = mw / s32;
    const int64_t bw = bw32, spw = mw - bw32 * s32;
    const int seg = (int)(tn / tiles_per_seg);  // the whole tile is Q (0), K (1) or V (2)
    const int hbase = (int)(tn - (uint32_t)seg * tiles_per_seg) * HEADS_PER_TILE;  // its first head
    const bool prologue = a.apply_prologue && seg < 2;
    float e_first = 1.f;  // exp(scale) of this warp's first head of the tile (Q tiles)
    if (prologue) {
      srow = a.sin + b * a.sin_b + sp * a.sin_n;
      crow = a.cos + b * a.cos_b + sp * a.cos_n;
#pragma unroll
      for (int g = 0; g < SLOTS; ++g) load_group(g, g);
      if (seg == 0) e_first = (float)exp((double)a.scales[hbase + head0]);
    }
    if (!mbar_wait(&sm.acc_full[abuf], (tcount >> 1) & 1)) break;
    tc_fence_after();
    const uint32_t tbase = tmem_base + abuf * kAccCols + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
    for (int hh = head0; hh < HEADS_PER_TILE; hh += HEAD_STEP) {
      const int h = hbase + hh;
      const uint32_t tcol = tbase + hh * D;
      const int64_t out_off = ((b * a.H + h) * a.S + sp) * D;
      const int64_t row0 = (bw * a.H + h) * a.S + spw;  // staged path: first output row
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out[seg]) + out_off;
      if (staged) reclaim();
      if (!prologue) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tcol + 32 * c, v);
          tmem_wait_ld();
          uint32_t p[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            p[i] = pack_bf16(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])));
#pragma unroll
          for (int q = 0; q < 4; ++q)
            emit16(out, valid, 32 * c + 8 * q, make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]));
        }
        if (staged) flush(&om.m[seg], row0);
        continue;
      }
      if (GROUPS > SLOTS && hh != head0) {
#pragma unroll
        for (int g = 0; g < SLOTS; ++g) load_group(g, g);
      }
      const float e = (seg == 0) ? (hh == head0 ? e_first : (float)exp((double)a.scales[h])) : 1.f;
      float sumsq;
      // Pass 1: BF16 projection (kept packed in registers for pass 2),
      // optional raw store, sum of squares; 32 columns per step, the next
      // step's TMEM loads in flight meanwhile.
      const bool want_raw = a.raw[seg] != nullptr;
      __nv_bfloat16* raw = want_raw ? static_cast<__nv_bfloat16*>(a.raw[seg]) + out_off : nullptr;
      uint32_t px[D / 2];  // px[i] = BF16 columns 2i, 2i + 1 of the head
      {
        float2 acc = make_float2(0.f, 0.f);
        uint32_t va[16], vb[16];  // one TMEM buffer: step c + 1 loads while step c's packed values are used
        tmem_ld16(tcol, va);
        tmem_ld16(tcol + 16, vb);
        tmem_wait_ld_regs(va, vb);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            px[16 * c + i] = pack_bf16(make_float2(__uint_as_float(va[2 * i]), __uint_as_float(va[2 * i + 1])));
            px[16 * c + 8 + i] = pack_bf16(make_float2(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1])));
          }
          if (c + 1 < D / 32) {
            tmem_ld16(tcol + 32 * (c + 1), va);
            tmem_ld16(tcol + 32 * (c + 1) + 16, vb);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 x = unpack_bf16(px[16 * c + i]);
            acc = __ffma2_rn(x, x, acc);  // squares of BF16 values are exact in FP32
          }
          if (want_raw) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              emit16(raw, valid, 32 * c + 8 * q,
                     make_uint4(px[16 * c + 4 * q], px[16 * c + 4 * q + 1], px[16 * c + 4 * q + 2], px[16 * c + 4 * q + 3]));
          }
          if (c + 1 < D / 32) tmem_wait_ld_regs(va, vb);
        }
        sumsq = __fadd_rn(acc.x, acc.y);
      }
      if (want_raw && staged) {
        flush(&om.m[3 + seg], row0);
        reclaim();
      }
      const float r = inv_rms<D>(sumsq, a.eps);
      const float2 r2 = splat2(r);
      const float2 e2 = splat2(e);
      const float* wrow = sm.w_s + seg * D;
      // Pass 2, 16 columns at a time from the registers of pass 1: columns j
      // and j + D/2 of the head are in this thread; each product and sum
      // rounds like the eager formulation.
#pragma unroll
      for (int g = 0; g < GROUPS; ++g) {
        const int slot = g % SLOTS;
        // The group's words are "defined" here for the compiler, so their
        // unpacking is not hoisted into earlier groups (which would hold every
        // column of the head unpacked at once and spill).
#pragma unroll
        for (int i = 0; i < 8; ++i) asm volatile("" : "+r"(px[8 * g + i]), "+r"(px[HALF / 2 + 8 * g + i]));
        uint32_t p1[8], p2[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const int j = 16 * g + 2 * i;  // column pair within the first half
          const float4 wa4 = *reinterpret_cast<const float4*>(wrow + j);
          const float4 wb4 = *reinterpret_cast<const float4*>(wrow + HALF + j);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float2 x1 = unpack_bf16(px[8 * g + i + u]);
            const float2 x2 = unpack_bf16(px[HALF / 2 + 8 * g + i + u]);
            const float2 wa = u ? make_float2(wa4.z, wa4.w) : make_float2(wa4.x, wa4.y);
            const float2 wb = u ? make_float2(wb4.z, wb4.w) : make_float2(wb4.x, wb4.y);
            const float2 c2 = make_float2(cs[slot][2 * (i + u)], cs[slot][2 * (i + u) + 1]);
            const float2 s2 = make_float2(sn[slot][2 * (i + u)], sn[slot][2 * (i + u) + 1]);
            const float2 y1 = __fmul2_rn(__fmul2_rn(x1, r2), wa);
            const float2 y2 = __fmul2_rn(__fmul2_rn(x2, r2), wb);
            float2 o1 = __fadd2_rn(__fmul2_rn(y1, c2), neg2(__fmul2_rn(y2, s2)));
            float2 o2 = __fadd2_rn(__fmul2_rn(y2, c2), __fmul2_rn(y1, s2));
            if (seg == 0) {
              o1 = __fmul2_rn(o1, e2);
              o2 = __fmul2_rn(o2, e2);
            }
            p1[i + u] = pack_bf16(o1);
            p2[i + u] = pack_bf16(o2);
          }
        }
        if (GROUPS > SLOTS && g + SLOTS < GROUPS) load_group(g + SLOTS, slot);
        emit16(out, valid, 16 * g, make_uint4(p1[0], p1[1], p1[2], p1[3]));
        emit16(out, valid, 16 * g + 8, make_uint4(p1[4], p1[5], p1[6], p1[7]));
        emit16(out, valid, HALF + 16 * g, make_uint4(p2[0], p2[1], p2[2], p2[3]));
        emit16(out, valid, HALF + 16 * g + 8, make_uint4(p2[4], p2[5], p2[6], p2[7]));
      }
      if (staged) flush(&om.m[seg], row0);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (ROWS == kRowsPair)
        mbar_arrive_cluster(acc_empty_cluster + abuf * (uint32_t)sizeof(uint64_t));
      else
        mbar_arrive(&sm.acc_empty[abuf]);
    }
  }
  // Every staged store must have completed before the CTA ends.
  if (staged && lane == 0) bulk_wait_group0();
}

// ---------------------------------------------------------------------------
// Single-CTA mainloop: one persistent CTA per SM, 128 x 256 tiles.
template <int D>
__global__ void __launch_bounds__(RolesSingle::kThreads, 1)
    qkv_gemm_prologue_kernel(const __grid_constant__ CUtensorMap tm_x,
                             const __grid_constant__ CUtensorMap tm_w,
                             const __grid_constant__ OutMaps om,
                             const __grid_constant__ GemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  using R = RolesSingle;
  const GemmSmem sm =
      carve_smem<kStagesSingle, kStageBytesSingle, kStagingBufsSingle, R::kEpi>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesSingle; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], R::kEpi);
    }
    mbar_init(sm.drain, 1);
    fence_mbar_init();
  }
  if (warp == R::kMma) {
    tmem_alloc(sm.tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (a.apply_prologue) {
    for (int i = threadIdx.x; i < 2 * D; i += R::kThreads) sm.w_s[i] = a.w[i];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *sm.tmem_slot;
  const int num_kb = (int)(a.K / BK);
  bool failed = false;

  if (warp == R::kProducer) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w);
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < a.n_tiles && !failed; tile += gridDim.x) {
        const int32_t m0 = (int32_t)((tile / a.n_tiles_n) * kRowsSingle);
        const int32_t n0 = (int32_t)((tile % a.n_tiles_n) * BN);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStagesSingle;
          if (!mbar_wait(&sm.empty[s], ((it / kStagesSingle) & 1) ^ 1)) { failed = true; break; }
          unsigned char* st = sm.ring + s * kStageBytesSingle;
          mbar_arrive_expect_tx(&sm.full[s], kStageBytesSingle);
          tma_load_2d(st, &tm_x, kb * BK, m0, &sm.full[s]);
          tma_load_2d(st + kStageASingle, &tm_w, kb * BK, n0, &sm.full[s]);
        }
      }
    }
  } else if (warp == R::kMma) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kRowsSingle, BN);
      uint32_t it = 0, tcount = 0;
      for (int64_t tile = blockIdx.x; tile < a.n_tiles && !failed; tile += gridDim.x, ++tcount) {
        const uint32_t abuf = tcount & 1;
        if (!mbar_wait(&sm.acc_empty[abuf], ((tcount >> 1) & 1) ^ 1)) { failed = true; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + abuf * kAccCols;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStagesSingle;
          if (!mbar_wait(&sm.full[s], (it / kStagesSingle) & 1)) { failed = true; break; }
          tc_fence_after();
          const uint32_t st = smem_u32(sm.ring + s * kStageBytesSingle);
          const uint64_t adesc = smem_desc_k_sw128(st);
          const uint64_t bdesc = smem_desc_k_sw128(st + kStageASingle);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // +32 bytes along K per step: +2 in the descriptor's start-address field.
            umma_bf16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          }
          umma_commit(&sm.empty[s]);  // releases the stage once these MMAs have read it
        }
        if (failed) break;
        umma_commit(&sm.acc_full[abuf]);
      }
      // Wait for the last accumulator's MMAs before TMEM may be released.
      if (tcount > 0 && !failed) {
        const uint32_t last = tcount - 1;
        mbar_wait(&sm.acc_full[last & 1], (last >> 1) & 1);
      }
      // A timed-out wait skipped that: wait (bounded) for every MMA issued so
      // far through one more commit, so TMEM is not released under them.
      if (failed && it > 0) {
        umma_commit(sm.drain);
        mbar_wait(sm.drain, 0);
      }
    }
  } else {
    run_epilogue<D, kRowsSingle, kStagingBufsSingle, R::kEpi, D / 32>(om, a, sm, tmem_base, blockIdx.x, gridDim.x, 0, 0u);
  }

  // Teardown: every warp arrives here (also after a timed-out wait).
  tc_fence_before();
  __syncthreads();
  if (warp == R::kMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair mainloop: 2-CTA clusters, 256 x 256 tiles (see the file comment).
template <int D, int EPI>
__global__ void __launch_bounds__(Roles<EPI>::kThreads, 1)
    qkv_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                         const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ OutMaps om,
                         const __grid_constant__ GemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  using C = PairConfig<EPI>;
  using R = typename C::R;
  constexpr int kStagesPair = C::kStages;
  const GemmSmem sm = carve_smem<kStagesPair, kStageBytesPair, kStagingBufsPair, R::kEpi>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the CTA that issues the MMAs
  const int64_t pair = blockIdx.x >> 1;
  const int64_t n_pairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesPair; ++s) {
      mbar_init(&sm.full[s], 1);   // even CTA: its producer's arrival + both CTAs' bytes
      mbar_init(&sm.empty[s], 1);  // one MMA commit per use, in each CTA
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 2 * R::kEpi);  // even CTA: the epilogue warps of both CTAs
    }
    mbar_init(sm.drain, 1);
    fence_mbar_init();
  }
  if (warp == R::kMma) {
    tmem_alloc_pair(sm.tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  if (a.apply_prologue) {
    for (int i = threadIdx.x; i < 2 * D; i += R::kThreads) sm.w_s[i] = a.w[i];
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *sm.tmem_slot;
  const int num_kb = (int)(a.K / BK);
  constexpr uint32_t kBar = sizeof(uint64_t);

  if (warp == R::kProducer) {
    // -------------------- TMA producer (both CTAs) --------------------
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w);
      const uint32_t full0 = mapa_shared(smem_u32(sm.full), 0);
      bool failed = false;
      uint32_t it = 0;
      for (int64_t tile = pair; tile < a.n_tiles && !failed; tile += n_pairs) {
        const int32_t m0 = (int32_t)((tile / a.n_tiles_n) * kRowsPair + rank * 128);
        const int32_t n0 = (int32_t)((tile % a.n_tiles_n) * BN + rank * (BN / 2));
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStagesPair;
          if (!mbar_wait(&sm.empty[s], ((it / kStagesPair) & 1) ^ 1)) { failed = true; break; }
          unsigned char* st = sm.ring + s * kStageBytesPair;
          if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], 2 * kStageBytesPair);
          tma_load_2d_pair(st, &tm_x, kb * BK, m0, full0 + s * kBar);
          tma_load_2d_pair(st + kStageAPair, &tm_w, kb * BK, n0, full0 + s * kBar);
        }
      }
      // Drain: wait until the MMA commits of the last uses of every stage have
      // arrived on this CTA's empty barriers, so none lands after the CTA ends.
      // (A stage never used passes at once: its wait is for the phase before the first.)
      for (int j = 0; j < kStagesPair && !failed; ++j, ++it) {
        const int s = it % kStagesPair;
        if (!mbar_wait(&sm.empty[s], ((it / kStagesPair) & 1) ^ 1)) failed = true;
      }
    }
  } else if (warp == R::kMma) {
    // -------------------- MMA issuer (even CTA, one thread) --------------------
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kRowsPair, BN);
      const uint32_t empty_own = mapa_shared(smem_u32(sm.empty), 0);
      const uint32_t empty_peer = mapa_shared(smem_u32(sm.empty), 1);
      const uint32_t accf_own = mapa_shared(smem_u32(sm.acc_full), 0);
      const uint32_t accf_peer = mapa_shared(smem_u32(sm.acc_full), 1);
      bool failed = false;
      uint32_t it = 0, tcount = 0;
      for (int64_t tile = pair; tile < a.n_tiles && !failed; tile += n_pairs, ++tcount) {
        const uint32_t abuf = tcount & 1;
        if (!mbar_wait_cluster(&sm.acc_empty[abuf], ((tcount >> 1) & 1) ^ 1)) { failed = true; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + abuf * kAccCols;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStagesPair;
          if (!mbar_wait(&sm.full[s], (it / kStagesPair) & 1)) { failed = true; break; }
          tc_fence_after();
          const uint32_t st = smem_u32(sm.ring + s * kStageBytesPair);
          const uint64_t adesc = smem_desc_k_sw128(st);
          const uint64_t bdesc = smem_desc_k_sw128(st + kStageAPair);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          // Release stage s in both CTAs once these MMAs have read it.
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
    run_epilogue<D, kRowsPair, kStagingBufsPair, R::kEpi, C::kSlots>(om, a, sm, tmem_base, pair, n_pairs, (int)rank * 128,
                               mapa_shared(smem_u32(sm.acc_empty), 0));
  }

  // Teardown: every thread of both CTAs arrives here (also after a timed-out
  // wait), so no CTA ends while its peer may still signal its barriers.
  tc_fence_before();
  __syncwarp();
  cluster_sync();
  if (warp == R::kMma) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side

namespace {

// 2-D BF16 row-major [rows, cols] map with a (64 x box_rows) box, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  const uint64_t dims[2] = {(uint64_t)cols, (uint64_t)rows};
  const uint64_t strides[1] = {(uint64_t)cols * 2};
  const uint32_t box[2] = {(uint32_t)BK, (uint32_t)box_rows};
  return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return sms;
}

template <int D>
cudaError_t launch_single(const CUtensorMap& mx, const CUtensorMap& mw, const OutMaps& om,
                          const GemmArgs& args, cudaStream_t stream) {
  const void* fn = reinterpret_cast<const void*>(&qkv_gemm_prologue_kernel<D>);
  const size_t smem = smem_bytes_for(kStagesSingle, kStageBytesSingle, kStagingBufsSingle,
                                     RolesSingle::kEpi, D);
  cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  const int sms = sm_count();
  if (sms <= 0) return cudaErrorInvalidDevice;
  const int64_t grid = args.n_tiles < sms ? args.n_tiles : sms;
  return launch_kernel(qkv_gemm_prologue_kernel<D>, dim3((unsigned)grid), dim3(RolesSingle::kThreads), smem,
                       stream, mx, mw, om, args);
}

// Co-resident 2-CTA clusters of a pair kernel on this device (cached).
template <int D, int EPI>
int resident_pairs(const cudaLaunchConfig_t& cfg) {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, qkv_gemm_pair_kernel<D, EPI>, &cfg) != cudaSuccess) return -1;
  if (dev < 64) cached[dev] = n;
  return n;
}

// Launch configuration of a pair kernel (grid set by the caller) and the
// number of its 2-CTA clusters that can be resident at once (0 if none can:
// the single-CTA mainloop is used then).
template <int D, int EPI>
int pair_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, cudaStream_t stream) {
  using C = PairConfig<EPI>;
  const size_t smem = smem_bytes_for(C::kStages, kStageBytesPair, kStagingBufsPair, EPI, D);
  if (cudaFuncSetAttribute(qkv_gemm_pair_kernel<D, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return 0;
  const int sms = sm_count();
  if (sms < 2) return 0;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3((unsigned)(sms & ~1));
  cfg->blockDim = dim3(C::R::kThreads);
  cfg->dynamicSmemBytes = smem;
  cfg->stream = stream;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
  const int n = resident_pairs<D, EPI>(*cfg);
  return n > 0 ? n : 0;
}

template <int D, int EPI>
cudaError_t launch_pair(const CUtensorMap& mx, const CUtensorMap& mw, const OutMaps& om,
                        const GemmArgs& args, cudaStream_t stream) {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  const int pairs_max = pair_config<D, EPI>(&cfg, attr, stream);
  if (pairs_max <= 0) return cudaErrorInvalidConfiguration;
  const int64_t pairs = args.n_tiles < pairs_max ? args.n_tiles : pairs_max;
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  return cudaLaunchKernelEx(&cfg, qkv_gemm_pair_kernel<D, EPI>, mx, mw, om, args);
}

// Which pair kernel serves this call (8 epilogue warps for the D = 128
// prologue: at D = 64 the 168-register budget of 10 warps would spill), and
// whether it can run here at all.
int pair_epilogue_warps(int64_t D, int apply_prologue) { return (apply_prologue && D == 128) ? 8 : 4; }

bool pair_runnable(int64_t D, int apply_prologue, cudaStream_t stream) {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  if (pair_epilogue_warps(D, apply_prologue) == 8) return pair_config<128, 8>(&cfg, attr, stream) > 0;
  return (D == 64 ? pair_config<64, 4>(&cfg, attr, stream) : pair_config<128, 4>(&cfg, attr, stream)) > 0;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 0: CTA-pair mainloop (default), 1: single-CTA mainloop.
int g_gemm_variant = 0;

}  // namespace

// The error word of this translation unit's bounded waits (tma_util.cuh).
cudaError_t read_gemm_device_error(int* value, bool reset) {
  cudaError_t err = cudaMemcpyFromSymbol(value, g_device_error, sizeof(int));
  if (err != cudaSuccess || !reset) return err;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
}

}  // namespace flash_prologue

using namespace flash_prologue;

extern "C" {

FLASH_PROLOGUE_API int flash_prologue_set_gemm_variant(int variant) {
  if (variant != 0 && variant != 1) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  g_gemm_variant = variant;
  return FLASH_PROLOGUE_OK;
}

FLASH_PROLOGUE_API int flash_prologue_qkv_gemm_fwd(
    const void* x, const void* w, int64_t M, int64_t K, int64_t H, int64_t D, int64_t S,
    const float* rmsnorm_weight, const float* scales, const float* sin,
    const int64_t sin_strides[3], const float* cos, const int64_t cos_strides[3], void* q_out,
    void* k_out, void* v_out, void* q_proj, void* k_proj, float eps, int apply_prologue,
    void* stream) {
  if (M < 0 || K <= 0 || H <= 0 || S <= 0) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (M == 0) return FLASH_PROLOGUE_OK;
  if (D != 64 && D != 128) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (K % BK != 0 || (H * D) % BN != 0 || M % S != 0) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (H > 512 || M * H >= (int64_t(1) << 31) || 3 * H * D >= (int64_t(1) << 31))
    return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (!x || !w || !q_out || !k_out || !v_out) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (!al16(x) || !al16(w) || !al16(q_out) || !al16(k_out) || !al16(v_out) ||
      (q_proj && !al16(q_proj)) || (k_proj && !al16(k_proj)))
    return FLASH_PROLOGUE_ERR_ALIGNMENT;
  if (apply_prologue) {
    if (!rmsnorm_weight || !scales || !sin || !cos || !sin_strides || !cos_strides)
      return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
    if (!(eps > 0.f) || !isfinite(eps)) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
    if (sin_strides[2] != 1 || cos_strides[2] != 1 || !al16(sin) || !al16(cos) ||
        ((sin_strides[0] | sin_strides[1] | cos_strides[0] | cos_strides[1]) & 3) != 0)
      return FLASH_PROLOGUE_ERR_ALIGNMENT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // CTA pairs unless selected off or the device cannot co-schedule 2-CTA clusters.
  const bool pair = g_gemm_variant == 0 && pair_runnable(D, apply_prologue, s);
  const int rows = pair ? kRowsPair : kRowsSingle;
  // Per CTA the pair loads 128 rows of X and 128 of W per stage; the single
  // CTA 128 rows of X and 256 of W.
  CUtensorMap mx, mw;
  if (!make_map(&mx, x, M, K, 128) || !make_map(&mw, w, 3 * H * D, K, pair ? BN / 2 : BN))
    return FLASH_PROLOGUE_ERR_CUDA;
  GemmArgs g{};
  g.M = M; g.K = K; g.H = H; g.D = D; g.S = S;
  g.n_tiles_n = 3 * H * D / BN;
  g.n_tiles = ((M + rows - 1) / rows) * g.n_tiles_n;
  g.w = rmsnorm_weight; g.scales = scales; g.sin = sin; g.cos = cos;
  if (apply_prologue) {
    g.sin_b = sin_strides[0]; g.sin_n = sin_strides[1];
    g.cos_b = cos_strides[0]; g.cos_n = cos_strides[1];
  }
  g.out[0] = q_out; g.out[1] = k_out; g.out[2] = v_out;
  g.raw[0] = q_proj; g.raw[1] = k_proj;
  g.eps = eps;
  g.apply_prologue = apply_prologue ? 1 : 0;
  // Outputs go through per-warp staging and TMA stores when every warp's 32
  // token rows are contiguous in [B, H, S, D] (S a multiple of 32).
  OutMaps om;
  g.tma_store = (S % 32 == 0) ? 1 : 0;
  if (g.tma_store) {
    void* outs[5] = {q_out, k_out, v_out, q_proj ? q_proj : q_out, k_proj ? k_proj : k_out};
    for (int i = 0; i < 5; ++i)
      if (!make_map(&om.m[i], outs[i], M * H, D, 32)) return FLASH_PROLOGUE_ERR_CUDA;
  } else {
    for (int i = 0; i < 5; ++i) om.m[i] = mx;  // unused
  }
  cudaError_t err;
  if (pair && pair_epilogue_warps(D, apply_prologue) == 8)
    err = launch_pair<128, 8>(mx, mw, om, g, s);
  else if (pair)
    err = (D == 64) ? launch_pair<64, 4>(mx, mw, om, g, s) : launch_pair<128, 4>(mx, mw, om, g, s);
  else
    err = (D == 64) ? launch_single<64>(mx, mw, om, g, s) : launch_single<128>(mx, mw, om, g, s);
  return err == cudaSuccess ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
}

}  // extern "C"
