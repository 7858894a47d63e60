// TMA pipelined forward and backward prologue kernels.
//
// CTA = 8 consumer warps + 1 producer warp, two CTAs per SM (the backward CTA
// has a whole producer warpgroup, which hands its registers to the consumers:
// kTmaBwdThreads in prologue_host.h). A tile is a block
// of rows of one batch b: `ti` consecutive rows along the "inner" row dim
// (heads for packed [T,H,D] views, positions for dense [B,H,N,D]), whose rows
// are contiguous in memory (inner stride == D), times `to` indices of the outer
// row dim. For every tile the producer warp issues one tiled TMA load per input
// tensor (a 5-D box that stores the tile's first half rows, then its second
// half rows: TmaTensor in prologue_host.h) plus one bulk copy per sin/cos table
// block, completing on the stage's full barrier. Consumer warps 0-3 process the
// Q rows of the stage, warps 4-7 the K rows: each lane owns one 16-element
// chunk pair of a row (the split-half RoPE partner of each element is in the
// same lane), reads it from shared memory without bank conflicts, and writes
// its results straight to global memory with 16-byte streaming stores. Stages
// are recycled through the empty barriers.
//
// The arithmetic per row is the one of the register-path kernels
// (prologue_fwd.cu / prologue_bwd.cu), in the same order, so both paths give
// bit-identical results.
#include <map>
#include <mutex>
#include <unordered_set>
#include <utility>

#include "prologue_host.h"
#include "tma_util.cuh"

namespace flash_prologue {

namespace {

template <typename T, int D>
struct TmaShape {
  static constexpr int ES = sizeof(T);
  static constexpr int ROW_BYTES = D * ES;
  static constexpr int ROWS = kTmaTileBytes / ROW_BYTES;        // rows per tensor per stage
  static constexpr int L = D / 16;                               // lanes per row
  static constexpr int LOG2_L = (L == 2) ? 1 : (L == 4) ? 2 : (L == 8) ? 3 : 4;
  static constexpr int HALF = D / 2;
  static constexpr int HALF_BYTES = HALF * ES;                   // a half row in shared memory
  static constexpr int HALF_TILE = ROWS * HALF_BYTES;            // first halves, then second halves
  static constexpr int GROUP_THREADS = kTmaConsumerWarps / 2 * 32;  // per tensor
  static constexpr int ROWS_PER_PASS = GROUP_THREADS / L;
  static constexpr int PASSES = ROWS / ROWS_PER_PASS;
  static_assert(PASSES >= 1 && ROWS % ROWS_PER_PASS == 0, "tile geometry");
};

struct TileCoords {
  int32_t b, i0, o0;  // batch, first inner row, first outer row
  int vi, vo;         // valid rows along inner / outer
};

// Tile of a cursor over (inner block, outer block, b); digit 3 flags the end.
__device__ __forceinline__ TileCoords tile_coords(const TmaPlan& p, const Cursor4& cur) {
  TileCoords tc;
  tc.b = cur.d[2];
  tc.i0 = cur.d[0] * p.ti;
  tc.o0 = cur.d[1] * p.to;
  const int64_t ri = p.inner_ext - (int64_t)tc.i0, ro = p.outer_ext - (int64_t)tc.o0;
  tc.vi = (int)(ri < p.ti ? ri : p.ti);
  tc.vo = (int)(ro < p.to ? ro : p.to);
  return tc;
}

// Issues the copies of one stage: lane t < nt loads streamed tensor t's tile
// with one tiled TMA load (rows outside the tensor read as zeros), lanes nt and
// nt + 1 copy the tile's sin and cos rows. Lane 0 has already armed the barrier.
template <int D>
__device__ __forceinline__ void issue_stage(const TmaTensor* in, int nt, const float* sin,
                                            const float* cos, int64_t sin_b, int64_t cos_b,
                                            int64_t n_first, int np, const TileCoords& tc,
                                            unsigned char* st, int table_bytes, uint64_t* bar,
                                            int lane, uint64_t pol_stream, uint64_t pol_table) {
  if (lane < nt) {
    tma_load_5d_hint(st + lane * kTmaTileBytes, &in[lane].map, 0, tc.i0, tc.o0, 0, tc.b, bar,
                     pol_stream);
  } else if (lane < nt + 2) {
    const bool is_cos = lane == nt + 1;
    const float* src = (is_cos ? cos : sin) + (int64_t)tc.b * (is_cos ? cos_b : sin_b) + n_first * (D / 2);
    bulk_g2s(st + nt * kTmaTileBytes + (is_cos ? table_bytes : 0), src, (uint32_t)np * (D / 2) * 4,
             bar, pol_table);
  }
}

// 8 values of the activation dtype from shared memory (16 or 32 bytes).
template <typename T>
__device__ __forceinline__ void lds_chunk(Chunk<T>& c, const unsigned char* p) {
  const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < Chunk<T>::kWords / 4; ++i) {
    const uint4 v = p4[i];
    c.w[4 * i + 0] = v.x; c.w[4 * i + 1] = v.y; c.w[4 * i + 2] = v.z; c.w[4 * i + 3] = v.w;
  }
}

__device__ __forceinline__ void lds_f8(float (&v)[kChunk], const unsigned char* p) {
  const float4* p4 = reinterpret_cast<const float4*>(p);
  const float4 a = p4[0], b = p4[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// 8 values of the activation dtype to shared memory (16 or 32 bytes).
template <typename T>
__device__ __forceinline__ void sts_chunk(unsigned char* p, const Chunk<T>& c) {
  uint4* p4 = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < Chunk<T>::kWords / 4; ++i)
    p4[i] = make_uint4(c.w[4 * i + 0], c.w[4 * i + 1], c.w[4 * i + 2], c.w[4 * i + 3]);
}

// Output tiles of one stage, which the consumers wrote over the stage's
// input tiles in the same half-major layout: lane t < 2 issues one tiled TMA
// store of tensor t's tile (rows outside the tensor are not written) and waits
// until the store has read shared memory, so the stage can be refilled.
__device__ __forceinline__ void store_stage_out(const TmaTensor* out, const unsigned char* st,
                                                int in_stride_tiles, const TileCoords& tc, int lane) {
  if (lane < 2) {
    tma_store_5d(&out[lane].map, st + lane * in_stride_tiles * kTmaTileBytes, 0, tc.i0, tc.o0, 0, tc.b);
    bulk_commit_group();
    bulk_wait_group_read0();
  }
  __syncwarp();
}

}  // namespace

// Forward that saves r: one tile's r values, staged by the consumers in the
// stage's r area ([tensor][row]), written by the producer warp to rms[t]
// ([B, H, N] FP32) with consecutive lanes on consecutive positions, so a warp
// store covers whole runs of a head's positions instead of one value per row.
template <int ROWS>
__device__ __forceinline__ void store_tile_r(const TmaFwdArgs& a, const TileCoords& tc,
                                             const float* r_s, int lane) {
  const int log2_to = __ffs(ROWS) - 1 - a.p.log2_ti;  // ti * to == ROWS, both powers of two
  for (int idx = lane; idx < 2 * ROWS; idx += 32) {
    const int t = idx >= ROWS;
    const int q = idx - t * ROWS;
    int i, o;  // inner / outer row index within the tile
    if (a.p.heads_inner) {
      o = q & ((1 << log2_to) - 1);
      i = q >> log2_to;
    } else {
      i = q & (a.p.ti - 1);
      o = q >> a.p.log2_ti;
    }
    if (o >= tc.vo || i >= tc.vi) continue;
    const int64_t h = a.p.heads_inner ? tc.i0 + i : tc.o0 + o;
    const int64_t n = a.p.heads_inner ? (int64_t)tc.o0 + o : (int64_t)tc.i0 + i;
    a.rms[t][((int64_t)tc.b * a.H + h) * a.N + n] = r_s[t * ROWS + (o << a.p.log2_ti) + i];
  }
}

// ---------------------------------------------------------------------------
// Forward. RMS = true also stores each row's r to a.rms (inverse formulation).
// TS = true writes q_out / k_out back into the stage's q / k tiles and lets the
// producer warp store them with TMA.
template <typename T, int D, bool RMS, bool TS>
__global__ void __launch_bounds__(kTmaThreads, 2)
    prologue_fwd_tma_kernel(const __grid_constant__ TmaFwdArgs a) {
  using S_ = TmaShape<T, D>;
  constexpr int HALF = S_::HALF;
  constexpr int L = S_::L;
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int S = kTmaFwdStages;  // == a.p.stages (the host plans with the same constant)
  const int table_bytes = a.p.P * HALF * 4;
  const int r_off = tma_stage_bytes(2, table_bytes);  // RMS: the tile's r values
  const int stage_bytes = r_off + (RMS ? tma_r_area_bytes(S_::ROWS) : 0);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;
  float* w_s = reinterpret_cast<float*>(empty + S);
  float* e_s = w_s + 2 * D;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTmaConsumerWarps);
    }
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 2 * D; i += kTmaThreads) w_s[i] = a.w[i];
  for (int i = threadIdx.x; i < a.H; i += kTmaThreads) e_s[i] = (float)exp((double)a.scales[i]);
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  Cursor4 cur;
  if (warp == kTmaConsumerWarps) {  // ---------------- producer ----------------
    const uint64_t pol_stream = policy_evict_normal();
    const uint64_t pol_table = policy_evict_last();
    int k = 0;
    bool failed = false;
    Cursor4 lag;  // RMS / TS: the tile whose r values / outputs go out next, S tiles behind
    lag.init(blockIdx.x, a.p.radix);
    for (cur.init(blockIdx.x, a.p.radix); cur.d[3] == 0; cur.advance(a.p.radix), ++k) {
      const int s = k % S;
      if (!mbar_wait(&empty[s], ((k / S) & 1) ^ 1)) { failed = true; break; }
      unsigned char* st = smem + s * stage_bytes;
      if ((RMS || TS) && k >= S) {  // the consumers are done with tile k - S
        const TileCoords lc = tile_coords(a.p, lag);
        if constexpr (RMS) store_tile_r<S_::ROWS>(a, lc, reinterpret_cast<const float*>(st + r_off), lane);
        if constexpr (TS) store_stage_out(a.out_map, st, 1, lc, lane);  // its outputs are in this stage
        lag.advance(a.p.radix);
      }
      const TileCoords tc = tile_coords(a.p, cur);
      const int64_t n_first = a.p.heads_inner ? (int64_t)tc.o0 : (int64_t)tc.i0;
      const int np = a.p.heads_inner ? tc.vo : tc.vi;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], 2 * kTmaTileBytes + 2 * np * HALF * 4);
      __syncwarp();
      issue_stage<D>(a.in, 2, a.sin, a.cos, a.sin_b, a.cos_b, n_first, np, tc, st, table_bytes,
                     &full[s], lane, pol_stream, pol_table);
    }
    if ((RMS || TS) && !failed) {  // r / outputs of the last (up to S) tiles, once the consumers are done
      for (int j = k > S ? k - S : 0; j < k; ++j) {
        const int s = j % S;
        if (!mbar_wait(&empty[s], (j / S) & 1)) break;
        const TileCoords lc = tile_coords(a.p, lag);
        const unsigned char* st = smem + s * stage_bytes;
        if constexpr (RMS) store_tile_r<S_::ROWS>(a, lc, reinterpret_cast<const float*>(st + r_off), lane);
        if constexpr (TS) store_stage_out(a.out_map, st, 1, lc, lane);
        lag.advance(a.p.radix);
      }
    }
    if constexpr (TS) {
      if (lane < 2) bulk_wait_group0();
    }
    return;
  }

  // ---------------- consumers: warps 0-3 Q, warps 4-7 K ----------------
  const int t = warp >> 2;
  const int gtid = threadIdx.x & (S_::GROUP_THREADS - 1);
  const int c = gtid & (L - 1);
  const int slot = gtid >> S_::LOG2_L;
  const int j0 = c * kChunk;
  const float* wa = w_s + t * D + j0;
  const float* wb = wa + HALF;
  T* yb = static_cast<T*>(a.out[t]);
  const RowStrides so = a.so[t];
  const int64_t so_inner = a.p.heads_inner ? so.h : so.n;
  const int64_t so_outer = a.p.heads_inner ? so.n : so.h;
  int k = 0;
  for (cur.init(blockIdx.x, a.p.radix); cur.d[3] == 0; cur.advance(a.p.radix), ++k) {
    const int s = k % S;
    if (!mbar_wait(&full[s], (k / S) & 1)) break;
    const TileCoords tc = tile_coords(a.p, cur);
    const unsigned char* st = smem + s * stage_bytes;
    const unsigned char* tile_x = st + t * kTmaTileBytes;
    const unsigned char* sin_s = st + 2 * kTmaTileBytes;
    const unsigned char* cos_s = sin_s + table_bytes;
    T* ytile = yb + (int64_t)tc.b * so.b + (int64_t)tc.i0 * so_inner + (int64_t)tc.o0 * so_outer + j0;
#pragma unroll
    for (int pass = 0; pass < S_::PASSES; ++pass) {
      const int r = pass * S_::ROWS_PER_PASS + slot;
      const int o_l = r >> a.p.log2_ti;
      const int i_l = r & (a.p.ti - 1);
      const bool ok = o_l < tc.vo && i_l < tc.vi;
      const unsigned char* row = tile_x + r * S_::HALF_BYTES + j0 * sizeof(T);
      Chunk<T> x1, x2;
      lds_chunk(x1, row);
      lds_chunk(x2, row + S_::HALF_TILE);
      const float ss = row_sum<L>(lane_sumsq(x1, x2));
      if (!ok) continue;
      const float rr = inv_rms<D>(ss, a.eps);
      const int p_l = a.p.heads_inner ? o_l : i_l;
      float sn[kChunk], cs[kChunk];
      lds_f8(sn, sin_s + (p_l * HALF + j0) * 4);
      lds_f8(cs, cos_s + (p_l * HALF + j0) * 4);
      const int h = a.p.heads_inner ? tc.i0 + i_l : tc.o0 + o_l;
      if (RMS && c == 0) reinterpret_cast<float*>(const_cast<unsigned char*>(st) + r_off)[t * S_::ROWS + r] = rr;
      Chunk<T> out1, out2;
      fwd_lane(x1, x2, rr, wa, wb, sn, cs, t == 0, t == 0 ? e_s[h] : 1.f, out1, out2);
      if constexpr (TS) {
        // Over this lane's own chunks of the q / k tile, read above.
        unsigned char* xw = const_cast<unsigned char*>(row);
        sts_chunk(xw, out1);
        sts_chunk(xw + S_::HALF_TILE, out2);
      } else {
        T* yp = ytile + (int64_t)i_l * so_inner + (int64_t)o_l * so_outer;
        store_stream<T, true>(yp, out1);
        store_stream<T, true>(yp + HALF, out2);
      }
    }
    if constexpr (TS) fence_proxy_async_smem();  // the producer's TMA stores read these tiles
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// ---------------------------------------------------------------------------
// Backward. INV = true is the inverse backward: the streamed "inputs" are the
// forward outputs, and each row's saved r is read from a.rms (prefetched
// before the stage's barrier wait so its latency overlaps the copy).
__device__ __forceinline__ float load_saved_r(const TmaBwdArgs& a, const TileCoords& tc, int t, int r) {
  const int o_l = r >> a.p.log2_ti;
  const int i_l = r & (a.p.ti - 1);
  if (o_l >= tc.vo || i_l >= tc.vi) return 0.f;
  const int64_t h = a.p.heads_inner ? (int64_t)tc.i0 + i_l : (int64_t)tc.o0 + o_l;
  const int64_t n = a.p.heads_inner ? (int64_t)tc.o0 + o_l : (int64_t)tc.i0 + i_l;
  return __ldg(a.rms[t] + ((int64_t)tc.b * a.H + h) * a.N + n);
}

// TS = true writes dq / dk back into the stage's q / k tiles (for the inverse
// backward: its q_out / k_out tiles) and lets the producer warp store them with
// TMA. Each lane overwrites only the chunks it has already read.
template <typename T, int D, bool INV, bool TS>
__global__ void __launch_bounds__(kTmaBwdThreads, 2)
    prologue_bwd_tma_kernel(const __grid_constant__ TmaBwdArgs a) {
  using S_ = TmaShape<T, D>;
  constexpr int HALF = S_::HALF;
  constexpr int L = S_::L;
  constexpr int LOG2_L = S_::LOG2_L;
  extern __shared__ __align__(128) unsigned char smem[];
  // Compile-time for the regular backward (2.4% faster at C2); the inverse
  // backward keeps the runtime value, whose division costs less there than
  // the register spill the constant caused (15% slower when measured).
  const int S = INV ? a.p.stages : kTmaBwdStages;  // == a.p.stages
  const int table_bytes = a.p.P * HALF * 4;
  const int stage_bytes = tma_stage_bytes(4, table_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;
  // w and 1 / w are read as float pairs (8-byte loads), so they come first,
  // at even offsets; the H-sized arrays, whose length may be odd, follow.
  float* w_s = reinterpret_cast<float*>(empty + S);   // [2 * D]
  float* iw_s = w_s + 2 * D;                           // INV: [2 * D] 1 / w
  float* e_s = iw_s + (INV ? 2 * D : 0);               // [H]
  float* ds_s = e_s + a.H;                             // [4][H]  (Q warps)
  float* dw_s = ds_s + 4 * a.H;                        // [8][D]
  float* ie_s = dw_s + 8 * D;                          // INV: [H] 1 / exp(scales)
  __shared__ int wait_failed;  // a consumer warp gave up on a barrier wait

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTmaConsumerWarps);
    }
    fence_mbar_init();
    wait_failed = 0;
  }
  for (int i = threadIdx.x; i < 2 * D; i += kTmaBwdThreads) w_s[i] = a.w[i];
  for (int i = threadIdx.x; i < a.H; i += kTmaBwdThreads) e_s[i] = (float)exp((double)a.scales[i]);
  for (int i = threadIdx.x; i < 4 * a.H; i += kTmaBwdThreads) ds_s[i] = 0.f;
  if constexpr (INV) {
    for (int i = threadIdx.x; i < 2 * D; i += kTmaBwdThreads) iw_s[i] = __frcp_rn(a.w[i]);
    for (int i = threadIdx.x; i < a.H; i += kTmaBwdThreads) ie_s[i] = (float)(1.0 / exp((double)a.scales[i]));
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  Cursor4 cur;
  if (warp >= kTmaConsumerWarps) {  // ---------------- producer warpgroup ----------------
    setmaxnreg_dec<kTmaBwdProducerRegs>();
    if (warp != kTmaConsumerWarps) return;
    const uint64_t pol_stream = policy_evict_normal();
    const uint64_t pol_table = policy_evict_last();
    int k = 0;
    bool failed = false;
    Cursor4 lag;  // TS: the tile whose outputs go out next, S tiles behind
    if constexpr (TS) lag.init(blockIdx.x, a.p.radix);
    for (cur.init(blockIdx.x, a.p.radix); cur.d[3] == 0; cur.advance(a.p.radix), ++k) {
      const int s = k % S;
      if (!mbar_wait(&empty[s], ((k / S) & 1) ^ 1)) { failed = true; break; }
      const TileCoords tc = tile_coords(a.p, cur);
      unsigned char* st = smem + s * stage_bytes;
      const int64_t n_first = a.p.heads_inner ? (int64_t)tc.o0 : (int64_t)tc.i0;
      const int np = a.p.heads_inner ? tc.vo : tc.vi;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], 4 * kTmaTileBytes + 2 * np * HALF * 4);
      __syncwarp();
      if constexpr (TS) {
        // The stage's gradient tiles and tables are free as soon as the
        // consumers are done: load them first (lanes 1, 3: gradient tiles;
        // 4, 5: tables), then store tile k - S's outputs from the q / k tiles,
        // and load the q / k tiles (lanes 0, 2) once the stores have read them.
        const bool early = (lane & 1) != 0 || lane >= 4;
        if (early)
          issue_stage<D>(a.in, 4, a.sin, a.cos, a.sin_b, a.cos_b, n_first, np, tc, st, table_bytes,
                         &full[s], lane, pol_stream, pol_table);
        if (k >= S) {
          store_stage_out(a.out, st, 2, tile_coords(a.p, lag), lane);
          lag.advance(a.p.radix);
        }
        if (!early)
          issue_stage<D>(a.in, 4, a.sin, a.cos, a.sin_b, a.cos_b, n_first, np, tc, st, table_bytes,
                         &full[s], lane, pol_stream, pol_table);
      } else {
        issue_stage<D>(a.in, 4, a.sin, a.cos, a.sin_b, a.cos_b, n_first, np, tc, st, table_bytes,
                       &full[s], lane, pol_stream, pol_table);
      }
    }
    if constexpr (TS) {
      if (!failed) {  // outputs of the last (up to S) tiles, once the consumers are done
        for (int j = k > S ? k - S : 0; j < k; ++j) {
          const int s = j % S;
          if (!mbar_wait(&empty[s], (j / S) & 1)) break;
          store_stage_out(a.out, smem + s * stage_bytes, 2, tile_coords(a.p, lag), lane);
          lag.advance(a.p.radix);
        }
      }
      if (lane < 2) bulk_wait_group0();
    }
    return;
  }

  // ---------------- consumers: warps 0-3 Q, warps 4-7 K ----------------
  setmaxnreg_inc<kTmaBwdConsumerRegs>();
  const int t = warp >> 2;
  const int gtid = threadIdx.x & (S_::GROUP_THREADS - 1);
  const int c = gtid & (L - 1);
  const int slot = gtid >> LOG2_L;
  const int j0 = c * kChunk;
  const float* wa = w_s + t * D + j0;
  const float* wb = wa + HALF;
  const float* iwa = iw_s + t * D + j0;
  const float* iwb = iwa + HALF;
  T* db = static_cast<T*>(a.dx[t]);
  const RowStrides sd = a.sd[t];
  const int64_t sd_inner = a.p.heads_inner ? sd.h : sd.n;
  const int64_t sd_outer = a.p.heads_inner ? sd.n : sd.h;

  // Lanes (within a warp) that hold rows of the same head differ only in the
  // chunk bits and in the lane bits [ps_lo, ps_hi).
  const int warp_slot_bits = 5 - LOG2_L;
  int ps_lo, ps_hi;
  if (a.p.heads_inner) {
    ps_lo = LOG2_L + min(a.p.log2_ti, warp_slot_bits);
    ps_hi = 5;
  } else {
    ps_lo = LOG2_L;
    ps_hi = LOG2_L + min(a.p.log2_ti, warp_slot_bits);
  }
  const bool ds_writer = ((lane & ((1 << ps_hi) - 1)) >> ps_lo) == 0 && c == 0;

  float2 acc1p[kPairs], acc2p[kPairs];  // d w partials for elements j0.. and HALF+j0..
#pragma unroll
  for (int q = 0; q < kPairs; ++q) { acc1p[q] = make_float2(0.f, 0.f); acc2p[q] = make_float2(0.f, 0.f); }

  static_assert(S_::PASSES <= 2, "saved-r prefetch holds two rows per thread");
  int k = 0;
  for (cur.init(blockIdx.x, a.p.radix); cur.d[3] == 0; cur.advance(a.p.radix), ++k) {
    const int s = k % S;
    const TileCoords tc = tile_coords(a.p, cur);
    float rv0 = 0.f, rv1 = 0.f;  // INV: saved r of this thread's rows in passes 0 and 1
    if constexpr (INV) {
      rv0 = load_saved_r(a, tc, t, slot);
      if (S_::PASSES > 1) rv1 = load_saved_r(a, tc, t, S_::ROWS_PER_PASS + slot);
    }
    if (!mbar_wait(&full[s], (k / S) & 1)) {
      wait_failed = 1;
      break;
    }
    const unsigned char* st = smem + s * stage_bytes;
    const unsigned char* tile_x = st + (2 * t) * kTmaTileBytes;
    const unsigned char* tile_g = st + (2 * t + 1) * kTmaTileBytes;
    const unsigned char* sin_s = st + 4 * kTmaTileBytes;
    const unsigned char* cos_s = sin_s + table_bytes;
    T* dtile = db + (int64_t)tc.b * sd.b + (int64_t)tc.i0 * sd_inner + (int64_t)tc.o0 * sd_outer + j0;
#pragma unroll
    for (int pass = 0; pass < S_::PASSES; ++pass) {
      const int r = pass * S_::ROWS_PER_PASS + slot;
      const int o_l = r >> a.p.log2_ti;
      const int i_l = r & (a.p.ti - 1);
      const bool ok = o_l < tc.vo && i_l < tc.vi;
      Chunk<T> x1, x2, g1, g2;
      float sn[kChunk], cs[kChunk];
      if (ok) {
        const unsigned char* xr = tile_x + r * S_::HALF_BYTES + j0 * sizeof(T);
        const unsigned char* gr = tile_g + r * S_::HALF_BYTES + j0 * sizeof(T);
        lds_chunk(x1, xr);
        lds_chunk(x2, xr + S_::HALF_TILE);
        lds_chunk(g1, gr);
        lds_chunk(g2, gr + S_::HALF_TILE);
        const int p_l = a.p.heads_inner ? o_l : i_l;
        lds_f8(sn, sin_s + (p_l * HALF + j0) * 4);
        lds_f8(cs, cos_s + (p_l * HALF + j0) * 4);
      } else {
#pragma unroll
        for (int q = 0; q < Chunk<T>::kWords; ++q) { x1.w[q] = 0; x2.w[q] = 0; g1.w[q] = 0; g2.w[q] = 0; }
#pragma unroll
        for (int j = 0; j < kChunk; ++j) { sn[j] = 0.f; cs[j] = 0.f; }
      }
      const int h = a.p.heads_inner ? tc.i0 + i_l : tc.o0 + o_l;
      const float e = (t == 0 && h < a.H) ? e_s[h] : 1.f;
      float2 dnw1[kPairs], dnw2[kPairs];  // u = d0 w (INV: t = d0 w)
      float2 n1[kPairs], n2[kPairs];      // n' = e n: x re, or rebuilt from the outputs (INV)
      float rr, re, dsum;
      if constexpr (INV) {
        rr = pass == 0 ? rv0 : rv1;
        re = __fmul_rn(rr, e);
        float part = 0.f;
        if (ok) {
          part = inv_lane_reduce(x1, x2, g1, g2, wa, wb, iwa, iwb, sn, cs, acc1p, acc2p, n1, n2, dnw1,
                                 dnw2);
        }
        dsum = row_sum<L>(part);
      } else {
        rr = inv_rms_bwd<D>(row_sum<L>(lane_sumsq2(x1, x2)), a.eps);
        re = __fmul_rn(rr, e);
        dsum = row_sum<L>(bwd_lane_reduce(x1, x2, g1, g2, re, wa, wb, sn, cs, acc1p, acc2p, dnw1,
                                          dnw2, n1, n2));
      }
      if (t == 0) {
        float v = dsum;
        for (int bit = ps_lo; bit < ps_hi; ++bit)
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1 << bit));
        if (ds_writer && h < a.H) ds_s[warp * a.H + h] += v;
      }
      if (!ok) continue;
      Chunk<T> out1, out2;
      if constexpr (INV)
        lane_dx<T>(n1, n2, dnw1, dnw2, re,
                       __fmul_rn(__fmul_rn(rr, dsum * (1.0f / (float)D)), t == 0 ? ie_s[h] : 1.f),
                       out1, out2);
      else
        lane_dx<T>(n1, n2, dnw1, dnw2, re, __fdividef(__fmul_rn(rr, dsum * (1.0f / (float)D)), e), out1,
                   out2);
      if constexpr (TS) {
        // Over this lane's own chunks of the q / k tile, read above.
        unsigned char* xw = const_cast<unsigned char*>(tile_x) + r * S_::HALF_BYTES + j0 * sizeof(T);
        sts_chunk(xw, out1);
        sts_chunk(xw + S_::HALF_TILE, out2);
      } else {
        T* dp = dtile + (int64_t)i_l * sd_inner + (int64_t)o_l * sd_outer;
        store_stream<T, true>(dp, out1);
        store_stream<T, true>(dp + HALF, out2);
      }
    }
    if constexpr (TS) fence_proxy_async_smem();  // the producer's TMA stores read these tiles
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // d w: combine lanes holding the same chunk (fixed xor order), then warps.
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
  consumer_sync(kTmaConsumerWarps * 32);
  // A CTA whose pipeline timed out has skipped tiles: its partial row is
  // written as NaN, so the parameter gradients the finalize kernel sums come
  // out NaN (besides the device error word) instead of silently short.
  const bool skipped = wait_failed != 0;
  const int C = 2 * D + a.H;
  float* out = a.partials + (int64_t)blockIdx.x * C;
  for (int col = threadIdx.x; col < C; col += kTmaConsumerWarps * 32) {
    float v = 0.f;
    if (col < D) {
#pragma unroll
      for (int w8 = 0; w8 < 4; ++w8) v = __fadd_rn(v, dw_s[w8 * D + col]);
    } else if (col < 2 * D) {
#pragma unroll
      for (int w8 = 4; w8 < 8; ++w8) v = __fadd_rn(v, dw_s[w8 * D + (col - D)]);
    } else {
#pragma unroll
      for (int w8 = 0; w8 < 4; ++w8) v = __fadd_rn(v, ds_s[w8 * a.H + (col - 2 * D)]);
    }
    out[col] = skipped ? __int_as_float(0x7fc00000) : v;
  }
}

// ---------------------------------------------------------------------------
// Self-test of the bounded-wait path: one thread waits on an mbarrier that
// nothing arrives at. After `tries` polls it gives up, records the timeout in
// this translation unit's error word (the word the pipelined kernels use) and
// returns, exactly as a protocol failure would; nothing faults or hangs.
__global__ void __launch_bounds__(32) selftest_wait_timeout_kernel(uint32_t tries) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const uint32_t a = smem_u32(&bar);
  for (uint32_t i = 0; i < tries; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(a), "r"(0u), "r"(kSuspendHintNs) : "memory");
    if (done) return;
  }
  atomicExch(&g_device_error, kDeviceErrorTimeout);
}

cudaError_t launch_selftest_wait_timeout(uint32_t tries, cudaStream_t stream) {
  return launch_kernel(selftest_wait_timeout_kernel, dim3(1), dim3(32), 0, stream, tries);
}

// ---------------------------------------------------------------------------
// Host side

cudaError_t read_device_error(int* value, bool reset) {
  cudaError_t err = cudaMemcpyFromSymbol(value, g_device_error, sizeof(int));
  if (err != cudaSuccess || !reset) return err;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
}

size_t tma_smem_bytes(const TmaPlan& p, int D, int n_tensors, int H, bool inv) {
  size_t stage = (size_t)tma_stage_bytes(n_tensors, p.P * (D / 2) * 4);
  if (n_tensors == 2 && inv) stage += (size_t)tma_r_area_bytes(p.ti * p.to);
  size_t extra = (size_t)2 * p.stages * sizeof(uint64_t) + (size_t)(2 * D + H) * 4;
  if (n_tensors == 4) extra += (size_t)(4 * H + 8 * D) * 4;
  if (inv) extra += (size_t)(2 * D + H) * 4;
  return p.stages * stage + extra;
}

template <typename T, int D>
static const void* fwd_tma_ptr(bool rms, bool ts) {
  if (rms)
    return ts ? reinterpret_cast<const void*>(&prologue_fwd_tma_kernel<T, D, true, true>)
              : reinterpret_cast<const void*>(&prologue_fwd_tma_kernel<T, D, true, false>);
  return ts ? reinterpret_cast<const void*>(&prologue_fwd_tma_kernel<T, D, false, true>)
            : reinterpret_cast<const void*>(&prologue_fwd_tma_kernel<T, D, false, false>);
}
template <typename T, int D>
static const void* bwd_tma_ptr(bool inv, bool ts) {
  if (inv)
    return ts ? reinterpret_cast<const void*>(&prologue_bwd_tma_kernel<T, D, true, true>)
              : reinterpret_cast<const void*>(&prologue_bwd_tma_kernel<T, D, true, false>);
  return ts ? reinterpret_cast<const void*>(&prologue_bwd_tma_kernel<T, D, false, true>)
            : reinterpret_cast<const void*>(&prologue_bwd_tma_kernel<T, D, false, false>);
}

// `inv`: the inverse backward, or for the forward the variant that stores r.
// `ts`: the variant whose outputs leave through TMA stores.
static const void* tma_kernel_for(bool bwd, int dtype, int D, bool inv, bool ts = false) {
#define FP_TMA_CASE(T)                                                                       \
  switch (D) {                                                                               \
    case 32: return bwd ? bwd_tma_ptr<T, 32>(inv, ts) : fwd_tma_ptr<T, 32>(inv, ts);         \
    case 64: return bwd ? bwd_tma_ptr<T, 64>(inv, ts) : fwd_tma_ptr<T, 64>(inv, ts);         \
    case 128: return bwd ? bwd_tma_ptr<T, 128>(inv, ts) : fwd_tma_ptr<T, 128>(inv, ts);      \
    case 256: return bwd ? bwd_tma_ptr<T, 256>(inv, ts) : fwd_tma_ptr<T, 256>(inv, ts);      \
    default: return nullptr;                                                                 \
  }
  switch (dtype) {
    case 0: FP_TMA_CASE(__nv_bfloat16)
    case 1: FP_TMA_CASE(__half)
    case 2: FP_TMA_CASE(float)
    default: return nullptr;
  }
#undef FP_TMA_CASE
}

// Opts the kernel in to `smem` bytes of dynamic shared memory on the current
// device. The attribute is per device and only has to grow, so the call is made
// once per (kernel, device) and larger size instead of on every launch.
static cudaError_t prepare_kernel(const void* fn, size_t smem) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> opted;
  const auto key = std::make_pair(fn, dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = opted.find(key);
    if (it != opted.end() && it->second >= smem) return cudaSuccess;
  }
  err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err == cudaSuccess) {
    std::lock_guard<std::mutex> lock(mu);
    size_t& v = opted[key];
    if (smem > v) v = smem;
  }
  return err;
}

// The backward kernel's register split (producer warpgroup down, consumers up)
// only completes if the kernel was built with at least kTmaBwdLaunchRegs
// registers per thread; a build with fewer is refused here instead of launched.
static cudaError_t check_bwd_registers(const void* fn) {
  static std::mutex mu;
  static std::unordered_set<const void*> checked;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (checked.count(fn)) return cudaSuccess;
  }
  cudaFuncAttributes attr;
  cudaError_t err = cudaFuncGetAttributes(&attr, fn);
  if (err != cudaSuccess) return err;
  if (attr.numRegs < kTmaBwdLaunchRegs) return cudaErrorInvalidConfiguration;
  std::lock_guard<std::mutex> lock(mu);
  checked.insert(fn);
  return cudaSuccess;
}

int64_t tma_grid(bool bwd, const TmaPlan& p, int H, int D, int dtype, bool inv) {
  const void* fn = tma_kernel_for(bwd, dtype, D, inv);
  if (!fn) return -1;
  const size_t smem = tma_smem_bytes(p, D, bwd ? 4 : 2, H, inv);
  if (prepare_kernel(fn, smem) != cudaSuccess) return -1;
  if (bwd && check_bwd_registers(fn) != cudaSuccess) return -1;
  return persistent_grid(fn, smem, p.n_tiles, bwd ? kTmaBwdThreads : kTmaThreads);
}

cudaError_t launch_fwd_tma(const TmaFwdArgs& a, int dtype, int D, cudaStream_t stream) {
  const void* fn = tma_kernel_for(false, dtype, D, a.rms[0] != nullptr, a.store_tma != 0);
  if (!fn) return cudaErrorInvalidValue;
  const size_t smem = tma_smem_bytes(a.p, D, 2, a.H, a.rms[0] != nullptr);
  cudaError_t err = prepare_kernel(fn, smem);
  if (err != cudaSuccess) return err;
  const int64_t grid = persistent_grid(fn, smem, a.p.n_tiles, kTmaThreads);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  TmaFwdArgs launch_args = a;
  launch_args.p.radix = make_radix(a.p.n_ib, a.p.n_ob, a.B, grid);
  void* args[] = {&launch_args};
  return cudaLaunchKernel(fn, dim3((unsigned)grid), dim3(kTmaThreads), args, smem, stream);
}

cudaError_t launch_bwd_tma(const TmaBwdArgs& a, float* dw, float* ds, int dtype, int D,
                           bool inv, const BwdReduce& red, cudaStream_t stream) {
  const void* fn = tma_kernel_for(true, dtype, D, inv, a.store_tma != 0);
  if (!fn) return cudaErrorInvalidValue;
  const size_t smem = tma_smem_bytes(a.p, D, 4, a.H, inv);
  cudaError_t err = prepare_kernel(fn, smem);
  if (err != cudaSuccess) return err;
  err = check_bwd_registers(fn);
  if (err != cudaSuccess) return err;
  const int64_t grid = persistent_grid(fn, smem, a.p.n_tiles, kTmaBwdThreads);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  TmaBwdArgs launch_args = a;
  launch_args.p.radix = make_radix(a.p.n_ib, a.p.n_ob, a.B, grid);
  void* args[] = {&launch_args};
  err = cudaLaunchKernel(fn, dim3((unsigned)grid), dim3(kTmaBwdThreads), args, smem, stream);
  if (err != cudaSuccess) return err;
  return launch_bwd_reduce(a.partials, grid, 2 * D + a.H, 2 * D, dw, ds, red, stream);
}

}  // namespace flash_prologue
