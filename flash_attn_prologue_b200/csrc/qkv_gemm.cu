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
// Structure (one persistent CTA per SM, 6 warps):
//   warp 4      TMA producer: 128x64 X tiles and 256x64 W tiles, 128-byte
//               swizzled, into a 4-stage shared-memory ring (full/empty mbarriers);
//   warp 5      allocates 512 TMEM columns; one thread issues tcgen05.mma
//               (M=128, N=256, K=16, BF16 -> FP32) into one of two TMEM
//               accumulators and commits stage releases / accumulator-ready;
//   warps 0-3   epilogue: tcgen05.ld of the accumulator (thread = token row),
//               BF16 rounding, sum of squares over the head, RoPE pairing of
//               columns j and j + D/2 (both in the same thread), stores.
// Double-buffered accumulators let the epilogue of tile i overlap the MMAs of
// tile i + 1. Tiles are ordered with the N tile fastest, so CTAs working at the
// same time share X rows through L2 (W stays L2-resident). All waits are
// bounded (tma_util.cuh); a timeout records an error, and TMEM is released on
// every path.
#include <cuda.h>

#include "../../include/flash_prologue.h"
#include "prologue_common.cuh"
#include "umma_util.cuh"

namespace flash_prologue {
namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 4;
constexpr int kStageA = BM * BK * 2;            // 16 KB
constexpr int kStageB = BN * BK * 2;            // 32 KB
constexpr int kStageBytes = kStageA + kStageB;  // 48 KB
constexpr int kAccCols = BN;                    // FP32 columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;         // two accumulators = all 512 columns
constexpr int kEpiWarps = 4;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kGemmThreads = (kEpiWarps + 2) * 32;
// Output staging: per epilogue warp, its 32 rows of one head as [32][128 B]
// halves (64 BF16 columns each), 128-byte swizzled, written out by TMA stores.
constexpr int kStageHalfBytes = 32 * 128;
constexpr int kStagingPerWarp = 2 * kStageHalfBytes;  // up to D = 128

struct GemmArgs {
  int64_t M, K, H, D, S;          // S = tokens per batch (M = B * S)
  int64_t n_tiles_n, n_tiles;
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

__device__ __forceinline__ float2 round_bf16_pair(uint32_t a, uint32_t b) {
  return __bfloat1622float2(__floats2bfloat162_rn(__uint_as_float(a), __uint_as_float(b)));
}

__device__ __forceinline__ uint32_t pack_bf16(float2 v) {
  __nv_bfloat162 p = __floats2bfloat162_rn(v.x, v.y);
  return *reinterpret_cast<uint32_t*>(&p);
}

// Stores 32 BF16 values (given as 16 packed words) as four 16-byte stores.
__device__ __forceinline__ void store32(__nv_bfloat16* dst, const uint32_t (&p)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
}

// Rounds one 32-column accumulator chunk to BF16 and stores it.
__device__ __forceinline__ void store_chunk_rounded(__nv_bfloat16* dst, const uint32_t (&v)[32]) {
  uint32_t p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) p[i] = pack_bf16(round_bf16_pair(v[2 * i], v[2 * i + 1]));
  store32(dst, p);
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

}  // namespace

template <int D>
__global__ void __launch_bounds__(kGemmThreads, 1)
    qkv_gemm_prologue_kernel(const __grid_constant__ CUtensorMap tm_x,
                             const __grid_constant__ CUtensorMap tm_w,
                             const __grid_constant__ OutMaps om,
                             const __grid_constant__ GemmArgs a) {
  constexpr int HALF = D / 2;
  constexpr int HEADS_PER_TILE = BN / D;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* staging = smem + kStages * kStageBytes;  // [kEpiWarps][kStagingPerWarp]
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + kEpiWarps * kStagingPerWarp);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* w_s = reinterpret_cast<float*>(tmem_slot + 4);  // [2 * D]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (a.apply_prologue) {
    for (int i = threadIdx.x; i < 2 * D; i += kGemmThreads) w_s[i] = a.w[i];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (int)(a.K / BK);
  bool failed = false;

  if (warp == kProducerWarp) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w);
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < a.n_tiles && !failed; tile += gridDim.x) {
        const int32_t m0 = (int32_t)((tile / a.n_tiles_n) * BM);
        const int32_t n0 = (int32_t)((tile % a.n_tiles_n) * BN);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1)) { failed = true; break; }
          unsigned char* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(st, &tm_x, kb * BK, m0, &full[s]);
          tma_load_2d(st + kStageA, &tm_w, kb * BK, n0, &full[s]);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      uint32_t it = 0, tcount = 0;
      for (int64_t tile = blockIdx.x; tile < a.n_tiles && !failed; tile += gridDim.x, ++tcount) {
        const uint32_t abuf = tcount & 1;
        if (!mbar_wait(&acc_empty[abuf], ((tcount >> 1) & 1) ^ 1)) { failed = true; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + abuf * kAccCols;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1)) { failed = true; break; }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * kStageBytes);
          const uint64_t adesc = smem_desc_k_sw128(st);
          const uint64_t bdesc = smem_desc_k_sw128(st + kStageA);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // +32 bytes along K per step: +2 in the descriptor's start-address field.
            umma_bf16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          }
          umma_commit(&empty[s]);  // releases the stage once these MMAs have read it
        }
        if (failed) break;
        umma_commit(&acc_full[abuf]);
      }
      // Wait for the last accumulator's MMAs before TMEM may be released.
      if (tcount > 0 && !failed) {
        const uint32_t last = tcount - 1;
        mbar_wait(&acc_full[last & 1], (last >> 1) & 1);
      }
    }
  } else {
    // ------------------------------ epilogue ----------------------------------
    const int row = warp * 32 + lane;  // TMEM lane == tile row
    unsigned char* stage_w = staging + warp * kStagingPerWarp;
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
    // Staged path: write the warp's 32 rows of one head to `map` at row0 ...
    auto flush = [&](const CUtensorMap* map, int64_t row0) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        for (int half = 0; half < D / 64; ++half)
          tma_store_2d(map, half * 64, (int32_t)row0, stage_w + half * kStageHalfBytes);
        bulk_commit_group();
      }
    };
    // ... and before refilling the staging tile, wait until those stores have read it.
    auto reclaim = [&]() {
      if (lane == 0) bulk_wait_group_read0();
      __syncwarp();
    };
    // The token's sin/cos row (D/2 + D/2 floats), fetched for every Q/K tile
    // before waiting for its accumulator so that the loads overlap the MMAs;
    // every head of the tile shares it.
    float sn[HALF], cs[HALF];
    uint32_t tcount = 0;
    for (int64_t tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x, ++tcount) {
      const uint32_t abuf = tcount & 1;
      const int64_t m = (tile / a.n_tiles_n) * BM + row;
      const bool valid = m < a.M;
      const int64_t b = m / a.S, sp = m % a.S;
      // First token of this warp's 32 rows (S % 32 == 0 on the staged path,
      // so all 32 share its batch index).
      const int64_t mw = (tile / a.n_tiles_n) * BM + warp * 32;
      const int64_t bw = mw / a.S, spw = mw % a.S;
      const int64_t n0 = (tile % a.n_tiles_n) * BN;
      const int seg = (int)(n0 / (a.H * D));  // the whole tile is Q (0), K (1) or V (2)
      const bool prologue = a.apply_prologue && seg < 2;
      if (prologue) {
        if (valid) {
          const float* srow = a.sin + b * a.sin_b + sp * a.sin_n;
          const float* crow = a.cos + b * a.cos_b + sp * a.cos_n;
#pragma unroll
          for (int j = 0; j < HALF; j += 4) {
            const float4 s4 = ldg4(srow + j), c4 = ldg4(crow + j);
            sn[j] = s4.x; sn[j + 1] = s4.y; sn[j + 2] = s4.z; sn[j + 3] = s4.w;
            cs[j] = c4.x; cs[j + 1] = c4.y; cs[j + 2] = c4.z; cs[j + 3] = c4.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < HALF; ++j) { sn[j] = 0.f; cs[j] = 0.f; }
        }
      }
      if (!mbar_wait(&acc_full[abuf], (tcount >> 1) & 1)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + abuf * kAccCols + ((uint32_t)(warp * 32) << 16);
      for (int hh = 0; hh < HEADS_PER_TILE; ++hh) {
        const int h = (int)(((n0 + hh * D) % (a.H * D)) / D);
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
            for (int i = 0; i < 16; ++i) p[i] = pack_bf16(round_bf16_pair(v[2 * i], v[2 * i + 1]));
#pragma unroll
            for (int q = 0; q < 4; ++q)
              emit16(out, valid, 32 * c + 8 * q, make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]));
          }
          if (staged) flush(&om.m[seg], row0);
          continue;
        }
        // Pass 1: BF16 projection, optional raw store, sum of squares.
        const bool want_raw = a.raw[seg] != nullptr;
        __nv_bfloat16* raw = want_raw ? static_cast<__nv_bfloat16*>(a.raw[seg]) + out_off : nullptr;
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tcol + 32 * c, v);
          tmem_wait_ld();
          uint32_t p[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 x = round_bf16_pair(v[2 * i], v[2 * i + 1]);
            acc = __ffma2_rn(x, x, acc);  // squares of BF16 values are exact in FP32
            p[i] = pack_bf16(x);
          }
          if (want_raw) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              emit16(raw, valid, 32 * c + 8 * q, make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]));
          }
        }
        if (want_raw && staged) {
          flush(&om.m[3 + seg], row0);
          reclaim();
        }
        const float r = inv_rms<D>(__fadd_rn(acc.x, acc.y), a.eps);
        const float2 r2 = splat2(r);
        const float2 e2 = splat2(seg == 0 ? (float)exp((double)a.scales[h]) : 1.f);
        const float* wrow = w_s + seg * D;
        // Pass 2, 16 columns at a time: columns j and j + D/2 of the head are
        // in this thread; each product and sum rounds like the eager formulation.
#pragma unroll
        for (int g = 0; g < HALF / 16; ++g) {
          uint32_t va[16], vb[16];
          tmem_ld16(tcol + 16 * g, va);
          tmem_ld16(tcol + HALF + 16 * g, vb);
          tmem_wait_ld();
          uint32_t p1[8], p2[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int j = 16 * g + 2 * i;  // column pair within the first half
            const float2 x1 = round_bf16_pair(va[2 * i], va[2 * i + 1]);
            const float2 x2 = round_bf16_pair(vb[2 * i], vb[2 * i + 1]);
            const float2 wa = ld_pair(wrow, j / 2);
            const float2 wb = ld_pair(wrow + HALF, j / 2);
            const float2 c2 = make_float2(cs[j], cs[j + 1]);
            const float2 s2 = make_float2(sn[j], sn[j + 1]);
            const float2 y1 = __fmul2_rn(__fmul2_rn(x1, r2), wa);
            const float2 y2 = __fmul2_rn(__fmul2_rn(x2, r2), wb);
            float2 o1 = __fadd2_rn(__fmul2_rn(y1, c2), neg2(__fmul2_rn(y2, s2)));
            float2 o2 = __fadd2_rn(__fmul2_rn(y2, c2), __fmul2_rn(y1, s2));
            if (seg == 0) {
              o1 = __fmul2_rn(o1, e2);
              o2 = __fmul2_rn(o2, e2);
            }
            p1[i] = pack_bf16(o1);
            p2[i] = pack_bf16(o2);
          }
          emit16(out, valid, 16 * g, make_uint4(p1[0], p1[1], p1[2], p1[3]));
          emit16(out, valid, 16 * g + 8, make_uint4(p1[4], p1[5], p1[6], p1[7]));
          emit16(out, valid, HALF + 16 * g, make_uint4(p2[0], p2[1], p2[2], p2[3]));
          emit16(out, valid, HALF + 16 * g + 8, make_uint4(p2[4], p2[5], p2[6], p2[7]));
        }
        if (staged) flush(&om.m[seg], row0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[abuf]);
    }
    // Every staged store must have completed before the CTA ends.
    if (staged && lane == 0) bulk_wait_group0();
  }

  // Teardown: every warp arrives here (also after a timed-out wait).
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D BF16 row-major [rows, cols] map with a (64 x box_rows) box, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t gemm_smem_bytes(int64_t D) {
  return 1024 + (size_t)kStages * kStageBytes + (size_t)kEpiWarps * kStagingPerWarp + 256 +
         (size_t)(2 * D) * 4;
}

template <int D>
cudaError_t launch_gemm(const CUtensorMap& mx, const CUtensorMap& mw, const OutMaps& om,
                        const GemmArgs& args, cudaStream_t stream) {
  const void* fn = reinterpret_cast<const void*>(&qkv_gemm_prologue_kernel<D>);
  const size_t smem = gemm_smem_bytes(D);
  cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  int dev = 0, sms = 0;
  if ((err = cudaGetDevice(&dev)) != cudaSuccess) return err;
  if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
  const int64_t grid = args.n_tiles < sms ? args.n_tiles : sms;
  qkv_gemm_prologue_kernel<D><<<(unsigned)grid, kGemmThreads, smem, stream>>>(mx, mw, om, args);
  return cudaGetLastError();
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

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
  CUtensorMap mx, mw;
  if (!make_map(&mx, x, M, K, BM) || !make_map(&mw, w, 3 * H * D, K, BN)) return FLASH_PROLOGUE_ERR_CUDA;
  GemmArgs g{};
  g.M = M; g.K = K; g.H = H; g.D = D; g.S = S;
  g.n_tiles_n = 3 * H * D / BN;
  g.n_tiles = ((M + BM - 1) / BM) * g.n_tiles_n;
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = (D == 64) ? launch_gemm<64>(mx, mw, om, g, s) : launch_gemm<128>(mx, mw, om, g, s);
  return err == cudaSuccess ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
}

}  // extern "C"
