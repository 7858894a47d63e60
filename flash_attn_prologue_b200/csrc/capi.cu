// C ABI of libflash_prologue.so: argument validation, layout planning and
// dispatch to the kernel launchers. Declarations: include/flash_prologue.h.
#include <math.h>

#include <mutex>
#include <unordered_map>

#include "../../include/flash_prologue.h"
#include "prologue_host.h"
#include "tensor_map.h"

namespace flash_prologue {

namespace {

int log2_exact(int64_t v) {
  int r = 0;
  while ((int64_t(1) << r) < v) ++r;
  return r;
}

int64_t pow2_floor(int64_t v) {
  int64_t p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace

Geometry plan_geometry(int64_t B, int64_t H, int64_t N, int D, bool heads_inner) {
  Geometry g{};
  const int L = D / 16;
  const int slots = kThreads / L;
  const int warp_slots = 32 / L;
  g.log2_l = log2_exact(L);
  g.heads_inner = heads_inner ? 1 : 0;
  int64_t hs, ps;
  if (heads_inner) {
    // Head slots along lanes: the largest power of two dividing H (no idle
    // lanes), unless that leaves a warp mostly spread over positions.
    hs = 1;
    while (hs * 2 <= slots && H % (hs * 2) == 0) hs *= 2;
    if (hs < 4 && hs < H) hs = pow2_floor(H < slots ? H : slots);
    ps = slots / hs;
    g.hi = (int)cdiv(H, hs);
  } else {
    ps = warp_slots >= 8 ? warp_slots : 8;
    if (ps > slots) ps = slots;
    hs = slots / ps;
    int64_t hi = cdiv(H, hs);
    g.hi = (int)(hi < 8 ? hi : 8);
  }
  g.log2_hs = log2_exact(hs);
  g.log2_ps = log2_exact(ps);
  g.n_pos_blocks = cdiv(N, ps);
  g.n_head_groups = cdiv(H, (int64_t)g.hi * hs);
  g.n_items = 2 * B * g.n_pos_blocks * g.n_head_groups;
  return g;
}

TmaPlan plan_tma(int64_t B, int64_t H, int64_t N, int D, int dtype, bool heads_inner, int stages) {
  TmaPlan p{};
  const int es = dtype == 2 ? 4 : 2;
  const int rows = kTmaTileBytes / (D * es);
  p.heads_inner = heads_inner ? 1 : 0;
  p.stages = stages;
  int64_t ti;
  if (heads_inner) {
    p.inner_ext = H;
    p.outer_ext = N;
    ti = 1;
    while (ti * 2 <= rows && H % (ti * 2) == 0) ti *= 2;
    if (ti < 4 && ti < H) ti = pow2_floor(H < rows ? H : rows);
  } else {
    p.inner_ext = N;
    p.outer_ext = H;
    ti = rows >= 16 ? rows / 4 : rows;
    if (N < ti) {
      int64_t c = 1;
      while (c < N) c *= 2;
      ti = c;
    }
  }
  p.ti = (int)ti;
  p.log2_ti = log2_exact(ti);
  p.to = (int)(rows / ti);
  p.P = heads_inner ? p.to : p.ti;
  p.n_ib = cdiv(p.inner_ext, p.ti);
  p.n_ob = cdiv(p.outer_ext, p.to);
  p.n_tiles = B * p.n_ob * p.n_ib;
  return p;
}

int64_t persistent_grid(const void* kernel, size_t smem_bytes, int64_t n_items, int threads) {
  struct Key {
    const void* fn;
    size_t smem;
    int dev;
    bool operator==(const Key& o) const { return fn == o.fn && smem == o.smem && dev == o.dev; }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.fn) ^ (k.smem * 1315423911u) ^ ((size_t)k.dev << 48);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, int64_t, KeyHash> cache;  // resident CTAs per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  Key key{kernel, smem_bytes, dev};
  int64_t resident = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) resident = it->second;
  }
  if (resident == 0) {
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem_bytes) !=
        cudaSuccess)
      return -1;
    if (per_sm < 1) per_sm = 1;
    resident = (int64_t)sms * per_sm;
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = resident;
  }
  return n_items < resident ? n_items : resident;
}

}  // namespace flash_prologue

using namespace flash_prologue;

namespace {

constexpr int64_t kMaxHeads = 512;

bool supported_dim(int64_t D) { return D == 32 || D == 64 || D == 128 || D == 256; }

size_t elem_size(int dtype) { return dtype == FLASH_PROLOGUE_FP32 ? 4 : 2; }

// Activation view checks: d stride 1, and no broadcast (stride 0) on a dim of size > 1.
int check_view(const int64_t s[4], int64_t B, int64_t H, int64_t N) {
  if (s[3] != 1) return FLASH_PROLOGUE_ERR_CHANNEL_STRIDE;
  if ((B > 1 && s[0] == 0) || (H > 1 && s[1] == 0) || (N > 1 && s[2] == 0))
    return FLASH_PROLOGUE_ERR_EXPANDED;
  return FLASH_PROLOGUE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 16-byte vector path: base 16-byte aligned and every row start 16-byte aligned.
bool view_vec_ok(const void* p, const int64_t s[4], size_t es) {
  if (!aligned16(p)) return false;
  for (int i = 0; i < 3; ++i)
    if (((s[i] * (int64_t)es) & 15) != 0) return false;
  return true;
}

bool table_vec_ok(const float* p, const int64_t s[3]) {
  if (!aligned16(p) || s[2] != 1) return false;
  return ((s[0] * 4) & 15) == 0 && ((s[1] * 4) & 15) == 0;
}

RowStrides rows(const int64_t s[4]) { return RowStrides{s[0], s[1], s[2]}; }
TableStrides table(const int64_t s[3]) { return TableStrides{s[0], s[1], s[2]}; }

bool heads_inner_layout(const int64_t s[4], int64_t H, int64_t N) {
  if (N == 1) return true;
  if (H == 1) return false;
  const int64_t sh = s[1] < 0 ? -s[1] : s[1];
  const int64_t sn = s[2] < 0 ? -s[2] : s[2];
  return sh <= sn;
}

int common_checks(const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                  const float* w, const float* sc, const float* sin, const int64_t* sins,
                  const float* cos, const int64_t* coss, int64_t B, int64_t H, int64_t N,
                  int64_t D, float eps, int dtype) {
  if (B < 0 || H < 0 || N < 0 || D <= 0) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (!(eps > 0.f) || !isfinite(eps)) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (dtype < 0 || dtype > 2 || !supported_dim(D)) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (H > kMaxHeads) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  // Work-cursor digits are 32-bit.
  if (B >= (int64_t(1) << 31) || N >= (int64_t(1) << 31)) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (!qs || !ks || !sins || !coss) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (B * H * N == 0) return FLASH_PROLOGUE_OK;
  if (!q || !k || !w || !sc || !sin || !cos) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  int st = check_view(qs, B, H, N);
  if (st == FLASH_PROLOGUE_OK) st = check_view(ks, B, H, N);
  return st;
}

// 0: automatic (TMA pipeline when the layout allows it, outputs stored as
// use_tma_stores picks), 1: register path only, 2: TMA pipeline with TMA-stored
// outputs wherever the output views allow, 3: TMA pipeline with the consumer
// lanes' stores.
int g_path_mode = 0;

constexpr int kFwdStages = kTmaFwdStages;
constexpr int kBwdStages = kTmaBwdStages;

// A streamed input the TMA path can read: 16-byte aligned, rows along the
// inner dim contiguous (stride D), positive b and outer strides that are
// 16-byte multiples, and a tensor map the driver accepts (the 5-D half-row
// view of TmaTensor, prologue_host.h). Dims of extent 1 get a placeholder
// stride (no address depends on it).
bool tma_tensor_ok(const void* p, const int64_t s[4], int64_t B, int64_t D, int dtype,
                   bool heads_inner, const TmaPlan& plan, TmaTensor* out) {
  const int64_t es = (int64_t)elem_size(dtype);
  if (!aligned16(p) || s[3] != 1) return false;
  const int64_t s_inner = heads_inner ? s[1] : s[2];
  const int64_t s_outer = heads_inner ? s[2] : s[1];
  if (s_inner != D) return false;
  const int64_t row = D * es;
  int64_t sb = s[0] * es, so = s_outer * es;
  if (B == 1) sb = row;
  if (plan.outer_ext == 1) so = row;
  if (sb <= 0 || so <= 0 || (sb & 15) != 0 || (so & 15) != 0) return false;
  const uint64_t dims[5] = {(uint64_t)(D / 2), (uint64_t)plan.inner_ext, (uint64_t)plan.outer_ext, 2,
                            (uint64_t)B};
  const uint64_t strides[4] = {(uint64_t)row, (uint64_t)so, (uint64_t)(row / 2), (uint64_t)sb};
  const uint32_t box[5] = {(uint32_t)(D / 2), (uint32_t)plan.ti, (uint32_t)plan.to, 2, 1};
  const CUtensorMapDataType type = dtype == 0   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  return encode_tensor_map(&out->map, type, 5, p, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// How the TMA kernels' outputs leave: written by the consumer lanes with 16-byte
// stores, or written back over the stage's input tiles and stored by the
// producer warp with one TMA tensor store per tile. Measured on B200 (paired,
// interleaved runs, identical bits): TMA stores take 0.956-0.978 of the lane
// stores' time in the D = 64 backward at every packed layout tested (0.992
// dense), and 0.95 in the D = 64 forward once each CTA streams about 900 tiles
// (neutral at 200-450, 1.04 slower at 110); at D = 128 they are 1.04-1.05
// (backward) and 1.12-1.15 (forward) slower. The inverse backward gains like
// the regular one (0.974-0.981 at D = 64); the forward that also saves r
// (`rms`) loses everywhere (1.13-1.19), its producer already writing the r
// values before it can refill a stage. `grid` is the forward's grid.
bool use_tma_stores(bool bwd, bool rms, int64_t D, const TmaPlan& p, int64_t grid) {
  if (g_path_mode == 2) return true;
  if (g_path_mode != 0 || D != 64) return false;
  return bwd || (!rms && grid > 0 && p.n_tiles >= 512 * grid);
}

// sin/cos tables the TMA path can read (bulk copies): rows of D/2 contiguous floats.
bool tma_table_ok(const float* p, const int64_t s[3], int64_t N, int64_t D) {
  if (!aligned16(p) || s[2] != 1) return false;
  if (N > 1 && s[1] != D / 2) return false;
  return ((s[0] * 4) & 15) == 0;
}

}  // namespace

extern "C" {

FLASH_PROLOGUE_API int flash_prologue_device_error(int* value, int reset) {
  if (!value) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  int a = 0, b = 0, c = 0, d = 0;
  if (read_device_error(&a, reset != 0) != cudaSuccess ||
      read_gemm_device_error(&b, reset != 0) != cudaSuccess ||
      read_gemm_bwd_device_error(&c, reset != 0) != cudaSuccess ||
      read_peer_device_error(&d, reset != 0) != cudaSuccess)
    return FLASH_PROLOGUE_ERR_CUDA;
  *value = a | b | c | d;
  return FLASH_PROLOGUE_OK;
}

FLASH_PROLOGUE_API int flash_prologue_selftest_wait_timeout(uint32_t tries, void* stream) {
  if (tries == 0 || tries > (1u << 22)) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  return launch_selftest_wait_timeout(tries, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? FLASH_PROLOGUE_OK
             : FLASH_PROLOGUE_ERR_CUDA;
}

FLASH_PROLOGUE_API int flash_prologue_set_path(int mode) {
  if (mode < 0 || mode > 3) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  g_path_mode = mode;
  return FLASH_PROLOGUE_OK;
}

const char* flash_prologue_status_string(int status) {
  switch (status) {
    case FLASH_PROLOGUE_OK: return "ok";
    case FLASH_PROLOGUE_ERR_INVALID_ARGUMENT: return "invalid argument (size, null pointer or eps)";
    case FLASH_PROLOGUE_ERR_UNSUPPORTED: return "unsupported head dimension, head count or dtype";
    case FLASH_PROLOGUE_ERR_CHANNEL_STRIDE: return "channel stride must be 1";
    case FLASH_PROLOGUE_ERR_EXPANDED: return "expanded activations (stride 0 on a dimension of size > 1) are not supported";
    case FLASH_PROLOGUE_ERR_WORKSPACE: return "workspace missing or too small";
    case FLASH_PROLOGUE_ERR_CUDA: return "CUDA launch or runtime error";
    case FLASH_PROLOGUE_ERR_ALIGNMENT: return "pointer alignment not supported";
    case FLASH_PROLOGUE_ERR_SCRATCH_LIMIT:
      return "problem needs more than the 1 MiB static scratch of flash_prologue_bwd_noalloc; "
             "use flash_prologue_bwd with a workspace";
    default: return "unknown status";
  }
}

int flash_prologue_version(void) { return 100; }

}  // extern "C"

namespace {

bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Forward; rms_q / rms_k (both null, or both FP32 [B, H, N]) receive r per row.
int fwd_impl(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
             void* q_out, const int64_t q_out_strides[4], void* k_out,
             const int64_t k_out_strides[4], float* rms_q, float* rms_k,
             const float* rmsnorm_weight, const float* scales, const float* sin,
             const int64_t sin_strides[3], const float* cos, const int64_t cos_strides[3],
             int64_t B, int64_t H, int64_t N, int64_t D, float eps, int dtype, void* stream) {
  int st = common_checks(q, q_strides, k, k_strides, rmsnorm_weight, scales, sin, sin_strides, cos,
                         cos_strides, B, H, N, D, eps, dtype);
  if (st != FLASH_PROLOGUE_OK || B * H * N == 0) return st;
  if (!q_out || !k_out || !q_out_strides || !k_out_strides) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if ((rms_q == nullptr) != (rms_k == nullptr)) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if ((rms_q && !aligned4(rms_q)) || (rms_k && !aligned4(rms_k))) return FLASH_PROLOGUE_ERR_ALIGNMENT;
  st = check_view(q_out_strides, B, H, N);
  if (st == FLASH_PROLOGUE_OK) st = check_view(k_out_strides, B, H, N);
  if (st != FLASH_PROLOGUE_OK) return st;

  const size_t es = elem_size(dtype);
  const bool vec = view_vec_ok(q, q_strides, es) && view_vec_ok(k, k_strides, es) &&
                   view_vec_ok(q_out, q_out_strides, es) && view_vec_ok(k_out, k_out_strides, es) &&
                   table_vec_ok(sin, sin_strides) && table_vec_ok(cos, cos_strides);
  const bool heads_inner = heads_inner_layout(q_strides, H, N);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g_path_mode != 1 && vec) {
    TmaFwdArgs t{};
    t.p = plan_tma(B, H, N, (int)D, dtype, heads_inner, kFwdStages);
    if (tma_tensor_ok(q, q_strides, B, D, dtype, heads_inner, t.p, &t.in[0]) &&
        tma_tensor_ok(k, k_strides, B, D, dtype, heads_inner, t.p, &t.in[1]) &&
        tma_table_ok(sin, sin_strides, N, D) && tma_table_ok(cos, cos_strides, N, D)) {
      t.out[0] = q_out; t.out[1] = k_out;
      t.so[0] = rows(q_out_strides); t.so[1] = rows(k_out_strides);
      t.store_tma = use_tma_stores(false, rms_q != nullptr, D, t.p,
                                   g_path_mode == 0 && D == 64 && !rms_q
                                       ? tma_grid(false, t.p, (int)H, (int)D, dtype, false)
                                       : 0) &&
                    tma_tensor_ok(q_out, q_out_strides, B, D, dtype, heads_inner, t.p, &t.out_map[0]) &&
                    tma_tensor_ok(k_out, k_out_strides, B, D, dtype, heads_inner, t.p, &t.out_map[1]);
      t.w = rmsnorm_weight; t.scales = scales; t.sin = sin; t.cos = cos;
      t.sin_b = sin_strides[0]; t.cos_b = cos_strides[0];
      t.rms[0] = rms_q; t.rms[1] = rms_k;
      t.B = B; t.N = N; t.H = (int)H; t.eps = eps;
      cudaError_t err = launch_fwd_tma(t, dtype, (int)D, s);
      return err == cudaSuccess ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
    }
  }
  FwdArgs a{};
  a.x[0] = q; a.x[1] = k; a.y[0] = q_out; a.y[1] = k_out;
  a.sx[0] = rows(q_strides); a.sx[1] = rows(k_strides);
  a.sy[0] = rows(q_out_strides); a.sy[1] = rows(k_out_strides);
  a.w = rmsnorm_weight; a.scales = scales; a.sin = sin; a.cos = cos;
  a.ssin = table(sin_strides); a.scos = table(cos_strides);
  a.rms[0] = rms_q; a.rms[1] = rms_k;
  a.B = B; a.N = N; a.H = (int)H; a.eps = eps;
  a.g = plan_geometry(B, H, N, (int)D, heads_inner);
  cudaError_t err = launch_fwd(a, dtype, (int)D, vec, s);
  return err == cudaSuccess ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
}

int bwd_plan(int64_t B, int64_t H, int64_t N, int64_t D, int dtype, bool vec, bool heads_inner,
             bool inv, Geometry* g, int64_t* grid) {
  *g = plan_geometry(B, H, N, (int)D, heads_inner);
  *grid = bwd_grid(*g, (int)H, (int)D, dtype, vec, inv);
  return *grid > 0 ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
}

}  // namespace

extern "C" {

int flash_prologue_fwd(const void* q, const int64_t q_strides[4], const void* k,
                       const int64_t k_strides[4], void* q_out, const int64_t q_out_strides[4],
                       void* k_out, const int64_t k_out_strides[4], const float* rmsnorm_weight,
                       const float* scales, const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3], int64_t B, int64_t H,
                       int64_t N, int64_t D, float eps, int dtype, void* stream) {
  return fwd_impl(q, q_strides, k, k_strides, q_out, q_out_strides, k_out, k_out_strides, nullptr,
                  nullptr, rmsnorm_weight, scales, sin, sin_strides, cos, cos_strides, B, H, N, D,
                  eps, dtype, stream);
}

int flash_prologue_inverse_fwd(const void* q, const int64_t q_strides[4], const void* k,
                               const int64_t k_strides[4], void* q_out,
                               const int64_t q_out_strides[4], void* k_out,
                               const int64_t k_out_strides[4], float* rms_q, float* rms_k,
                               const float* rmsnorm_weight, const float* scales, const float* sin,
                               const int64_t sin_strides[3], const float* cos,
                               const int64_t cos_strides[3], int64_t B, int64_t H, int64_t N,
                               int64_t D, float eps, int dtype, void* stream) {
  if (B * H * N > 0 && (!rms_q || !rms_k)) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  return fwd_impl(q, q_strides, k, k_strides, q_out, q_out_strides, k_out, k_out_strides, rms_q,
                  rms_k, rmsnorm_weight, scales, sin, sin_strides, cos, cos_strides, B, H, N, D,
                  eps, dtype, stream);
}

int flash_prologue_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D, int dtype,
                                      size_t* bytes) {
  if (!bytes) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  *bytes = 0;
  if (B < 0 || H < 0 || N < 0) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (dtype < 0 || dtype > 2 || !supported_dim(D) || H > kMaxHeads) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (B >= (int64_t(1) << 31) || N >= (int64_t(1) << 31)) return FLASH_PROLOGUE_ERR_UNSUPPORTED;
  if (B * H * N == 0) return FLASH_PROLOGUE_OK;
  // The grid (and so the workspace) is the largest of the layouts and vector
  // widths the call may pick, so one size serves every stride pattern.
  // The inverse backward's kernels are included, so the same size serves
  // flash_prologue_inverse_bwd.
  int64_t worst = 0;
  for (int inv = 0; inv < 2; ++inv) {
    for (int hi = 0; hi < 2; ++hi) {
      for (int v = 0; v < 2; ++v) {
        Geometry g;
        int64_t grid;
        int st = bwd_plan(B, H, N, D, dtype, v != 0, hi != 0, inv != 0, &g, &grid);
        if (st != FLASH_PROLOGUE_OK) return st;
        if (grid > worst) worst = grid;
      }
      const int64_t tgrid = tma_grid(true, plan_tma(B, H, N, D, dtype, hi != 0, kBwdStages),
                                     (int)H, (int)D, dtype, inv != 0);
      if (tgrid <= 0) return FLASH_PROLOGUE_ERR_CUDA;
      if (tgrid > worst) worst = tgrid;
    }
  }
  *bytes = (size_t)worst * (size_t)(2 * D + H) * sizeof(float);
  return FLASH_PROLOGUE_OK;
}

}  // extern "C"

namespace {

// Backward. With inv, q / k are the forward outputs and rms_q / rms_k their saved r.
int bwd_impl(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
             const float* rms_q, const float* rms_k, bool inv, const float* rmsnorm_weight,
             const float* scales, const float* sin, const int64_t sin_strides[3], const float* cos,
             const int64_t cos_strides[3], const void* grad_q_out, const int64_t gq_strides[4],
             const void* grad_k_out, const int64_t gk_strides[4], void* grad_q,
             const int64_t dq_strides[4], void* grad_k, const int64_t dk_strides[4],
             float* grad_rmsnorm_weight, float* grad_scales, void* workspace,
             size_t workspace_bytes, int64_t B, int64_t H, int64_t N, int64_t D, float eps,
             int dtype, void* stream, const BwdReduce& red = BwdReduce{}) {
  int st = common_checks(q, q_strides, k, k_strides, rmsnorm_weight, scales, sin, sin_strides, cos,
                         cos_strides, B, H, N, D, eps, dtype);
  if (st != FLASH_PROLOGUE_OK) return st;
  if (!grad_rmsnorm_weight || !grad_scales) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (red.peers && B * H * N == 0) return FLASH_PROLOGUE_ERR_UNSUPPORTED;  // every rank must add rows
  if (B * H * N == 0) {
    // No rows: the parameter gradients are exactly zero.
    if (cudaMemsetAsync(grad_rmsnorm_weight, 0, sizeof(float) * 2 * D, s) != cudaSuccess ||
        (H > 0 && cudaMemsetAsync(grad_scales, 0, sizeof(float) * H, s) != cudaSuccess))
      return FLASH_PROLOGUE_ERR_CUDA;
    return FLASH_PROLOGUE_OK;
  }
  if (!grad_q_out || !grad_k_out || !grad_q || !grad_k || !gq_strides || !gk_strides ||
      !dq_strides || !dk_strides)
    return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  if (inv) {
    if (!rms_q || !rms_k) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
    if (!aligned4(rms_q) || !aligned4(rms_k)) return FLASH_PROLOGUE_ERR_ALIGNMENT;
  }
  // Upstream gradients are only read, so broadcast (stride-0) views such as the
  // gradient of a sum() are read in place; their d stride must still be 1.
  if (gq_strides[3] != 1 || gk_strides[3] != 1) return FLASH_PROLOGUE_ERR_CHANNEL_STRIDE;
  st = check_view(dq_strides, B, H, N);
  if (st == FLASH_PROLOGUE_OK) st = check_view(dk_strides, B, H, N);
  if (st != FLASH_PROLOGUE_OK) return st;

  const size_t es = elem_size(dtype);
  const bool vec = view_vec_ok(q, q_strides, es) && view_vec_ok(k, k_strides, es) &&
                   view_vec_ok(grad_q_out, gq_strides, es) && view_vec_ok(grad_k_out, gk_strides, es) &&
                   view_vec_ok(grad_q, dq_strides, es) && view_vec_ok(grad_k, dk_strides, es) &&
                   table_vec_ok(sin, sin_strides) && table_vec_ok(cos, cos_strides);
  const bool heads_inner = heads_inner_layout(q_strides, H, N);
  if (g_path_mode != 1 && vec) {
    TmaBwdArgs t{};
    t.p = plan_tma(B, H, N, (int)D, dtype, heads_inner, kBwdStages);
    if (tma_tensor_ok(q, q_strides, B, D, dtype, heads_inner, t.p, &t.in[0]) &&
        tma_tensor_ok(grad_q_out, gq_strides, B, D, dtype, heads_inner, t.p, &t.in[1]) &&
        tma_tensor_ok(k, k_strides, B, D, dtype, heads_inner, t.p, &t.in[2]) &&
        tma_tensor_ok(grad_k_out, gk_strides, B, D, dtype, heads_inner, t.p, &t.in[3]) &&
        tma_table_ok(sin, sin_strides, N, D) && tma_table_ok(cos, cos_strides, N, D)) {
      const int64_t tgrid = tma_grid(true, t.p, (int)H, (int)D, dtype, inv);
      if (tgrid <= 0) return FLASH_PROLOGUE_ERR_CUDA;
      const size_t tneed = (size_t)tgrid * (size_t)(2 * D + H) * sizeof(float);
      if (!workspace || workspace_bytes < tneed || !aligned16(workspace))
        return FLASH_PROLOGUE_ERR_WORKSPACE;
      t.dx[0] = grad_q; t.dx[1] = grad_k;
      t.sd[0] = rows(dq_strides); t.sd[1] = rows(dk_strides);
      t.store_tma = use_tma_stores(true, false, D, t.p, 0) &&
                    tma_tensor_ok(grad_q, dq_strides, B, D, dtype, heads_inner, t.p, &t.out[0]) &&
                    tma_tensor_ok(grad_k, dk_strides, B, D, dtype, heads_inner, t.p, &t.out[1]);
      t.w = rmsnorm_weight; t.scales = scales; t.sin = sin; t.cos = cos;
      t.sin_b = sin_strides[0]; t.cos_b = cos_strides[0];
      t.partials = static_cast<float*>(workspace);
      t.rms[0] = rms_q; t.rms[1] = rms_k;
      t.B = B; t.N = N; t.H = (int)H; t.eps = eps;
      cudaError_t err = launch_bwd_tma(t, grad_rmsnorm_weight, grad_scales, dtype, (int)D, inv, red, s);
      return err == cudaSuccess ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
    }
  }
  Geometry g;
  int64_t grid;
  st = bwd_plan(B, H, N, D, dtype, vec, heads_inner, inv, &g, &grid);
  if (st != FLASH_PROLOGUE_OK) return st;
  const size_t need = (size_t)grid * (size_t)(2 * D + H) * sizeof(float);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) return FLASH_PROLOGUE_ERR_WORKSPACE;

  BwdArgs a{};
  a.x[0] = q; a.x[1] = k; a.gy[0] = grad_q_out; a.gy[1] = grad_k_out;
  a.dx[0] = grad_q; a.dx[1] = grad_k;
  a.sx[0] = rows(q_strides); a.sx[1] = rows(k_strides);
  a.sgy[0] = rows(gq_strides); a.sgy[1] = rows(gk_strides);
  a.sdx[0] = rows(dq_strides); a.sdx[1] = rows(dk_strides);
  a.w = rmsnorm_weight; a.scales = scales; a.sin = sin; a.cos = cos;
  a.ssin = table(sin_strides); a.scos = table(cos_strides);
  a.partials = static_cast<float*>(workspace);
  a.rms[0] = rms_q; a.rms[1] = rms_k;
  a.B = B; a.N = N; a.H = (int)H; a.eps = eps;
  a.g = g;
  cudaError_t err = launch_bwd(a, grad_rmsnorm_weight, grad_scales, dtype, (int)D, vec, inv, red, s);
  return err == cudaSuccess ? FLASH_PROLOGUE_OK : FLASH_PROLOGUE_ERR_CUDA;
}

// The reduction of a data-parallel backward: a valid group (its rank inside it,
// a row long enough for 2 * D + H sums, a wait bound within limits) and an epoch
// of at least 1.
bool peer_reduce_of(const flash_prologue_peers* peers, uint32_t epoch, int64_t D, int64_t H, BwdReduce* red) {
  if (!peers || epoch == 0) return false;
  if (peers->world < 1 || peers->world > FLASH_PROLOGUE_MAX_PEERS || peers->rank < 0 ||
      peers->rank >= peers->world || peers->max_cols % 32 != 0 || peers->max_cols < 2 * D + H ||
      peers->wait_ms < 0 || peers->wait_ms > 60000)
    return false;
  red->peers = peers;
  red->epoch = epoch;
  return true;
}

}  // namespace

extern "C" {

int flash_prologue_bwd(const void* q, const int64_t q_strides[4], const void* k,
                       const int64_t k_strides[4], const float* rmsnorm_weight,
                       const float* scales, const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3], const void* grad_q_out,
                       const int64_t gq_strides[4], const void* grad_k_out,
                       const int64_t gk_strides[4], void* grad_q, const int64_t dq_strides[4],
                       void* grad_k, const int64_t dk_strides[4], float* grad_rmsnorm_weight,
                       float* grad_scales, void* workspace, size_t workspace_bytes, int64_t B,
                       int64_t H, int64_t N, int64_t D, float eps, int dtype, void* stream) {
  return bwd_impl(q, q_strides, k, k_strides, nullptr, nullptr, false, rmsnorm_weight, scales, sin,
                  sin_strides, cos, cos_strides, grad_q_out, gq_strides, grad_k_out, gk_strides,
                  grad_q, dq_strides, grad_k, dk_strides, grad_rmsnorm_weight, grad_scales,
                  workspace, workspace_bytes, B, H, N, D, eps, dtype, stream);
}

int flash_prologue_bwd_dp(const void* q, const int64_t q_strides[4], const void* k,
                          const int64_t k_strides[4], const float* rmsnorm_weight, const float* scales,
                          const float* sin, const int64_t sin_strides[3], const float* cos,
                          const int64_t cos_strides[3], const void* grad_q_out, const int64_t gq_strides[4],
                          const void* grad_k_out, const int64_t gk_strides[4], void* grad_q,
                          const int64_t dq_strides[4], void* grad_k, const int64_t dk_strides[4],
                          float* grad_rmsnorm_weight, float* grad_scales, void* workspace,
                          size_t workspace_bytes, int64_t B, int64_t H, int64_t N, int64_t D, float eps,
                          int dtype, const flash_prologue_peers* peers, uint32_t epoch, void* stream) {
  BwdReduce red;
  if (!peer_reduce_of(peers, epoch, D, H, &red)) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  return bwd_impl(q, q_strides, k, k_strides, nullptr, nullptr, false, rmsnorm_weight, scales, sin,
                  sin_strides, cos, cos_strides, grad_q_out, gq_strides, grad_k_out, gk_strides,
                  grad_q, dq_strides, grad_k, dk_strides, grad_rmsnorm_weight, grad_scales,
                  workspace, workspace_bytes, B, H, N, D, eps, dtype, stream, red);
}

int flash_prologue_inverse_bwd_dp(const void* q_out, const int64_t q_out_strides[4],
                                  const void* k_out, const int64_t k_out_strides[4],
                                  const float* rms_q, const float* rms_k,
                                  const float* rmsnorm_weight, const float* scales, const float* sin,
                                  const int64_t sin_strides[3], const float* cos,
                                  const int64_t cos_strides[3], const void* grad_q_out,
                                  const int64_t gq_strides[4], const void* grad_k_out,
                                  const int64_t gk_strides[4], void* grad_q,
                                  const int64_t dq_strides[4], void* grad_k,
                                  const int64_t dk_strides[4], float* grad_rmsnorm_weight,
                                  float* grad_scales, void* workspace, size_t workspace_bytes,
                                  int64_t B, int64_t H, int64_t N, int64_t D, float eps, int dtype,
                                  const flash_prologue_peers* peers, uint32_t epoch, void* stream) {
  BwdReduce red;
  if (!peer_reduce_of(peers, epoch, D, H, &red)) return FLASH_PROLOGUE_ERR_INVALID_ARGUMENT;
  return bwd_impl(q_out, q_out_strides, k_out, k_out_strides, rms_q, rms_k, true, rmsnorm_weight,
                  scales, sin, sin_strides, cos, cos_strides, grad_q_out, gq_strides, grad_k_out,
                  gk_strides, grad_q, dq_strides, grad_k, dk_strides, grad_rmsnorm_weight,
                  grad_scales, workspace, workspace_bytes, B, H, N, D, eps, dtype, stream, red);
}

int flash_prologue_inverse_bwd(const void* q_out, const int64_t q_out_strides[4],
                               const void* k_out, const int64_t k_out_strides[4],
                               const float* rms_q, const float* rms_k,
                               const float* rmsnorm_weight, const float* scales, const float* sin,
                               const int64_t sin_strides[3], const float* cos,
                               const int64_t cos_strides[3], const void* grad_q_out,
                               const int64_t gq_strides[4], const void* grad_k_out,
                               const int64_t gk_strides[4], void* grad_q,
                               const int64_t dq_strides[4], void* grad_k,
                               const int64_t dk_strides[4], float* grad_rmsnorm_weight,
                               float* grad_scales, void* workspace, size_t workspace_bytes,
                               int64_t B, int64_t H, int64_t N, int64_t D, float eps, int dtype,
                               void* stream) {
  return bwd_impl(q_out, q_out_strides, k_out, k_out_strides, rms_q, rms_k, true, rmsnorm_weight,
                  scales, sin, sin_strides, cos, cos_strides, grad_q_out, gq_strides, grad_k_out,
                  gk_strides, grad_q, dq_strides, grad_k, dk_strides, grad_rmsnorm_weight,
                  grad_scales, workspace, workspace_bytes, B, H, N, D, eps, dtype, stream);
}

}  // extern "C"
