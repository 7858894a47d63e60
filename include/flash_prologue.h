/*
 * flash_prologue.h -- C ABI of the B200 (sm_100a) attention-prologue library
 * (libflash_prologue.so).
 *
 * The op ("qknorm_rope_scale") is, per (batch b, head h, position n) row of
 * length D:
 *     r      = 1 / sqrt(mean_j(x_j^2) + eps)              (FP32)
 *     y_j    = (x_j * r) * w[t][j]                        t = 0 for Q, 1 for K
 *     o_j    = y_j * cos_j - y_{j+D/2} * sin_j            j <  D/2
 *     o_{j+D/2} = y_{j+D/2} * cos_j + y_j * sin_j
 *     Q only: o *= exp(scales[h])
 *     out    = cast(o) to the input dtype (once)
 * with sin/cos FP32 tables indexed by (b, n) and shared by every head.
 *
 * Conventions shared by every entry point:
 *   - Activations are 4-D [B, H, N, D] views given by a base pointer and four
 *     int64 strides in ELEMENTS, ordered (b, h, n, d). The d stride must be 1.
 *     A packed [T, H, D] tensor is passed as B=1, N=T with strides
 *     (0, stride_h, stride_t, 1), so strided views into a fused QKV buffer
 *     need no copy.
 *   - sin/cos are FP32 and indexed [b, n, j] (j < D/2) through three strides
 *     (b, n, j) in elements; a stride of 0 broadcasts that dimension.
 *   - rmsnorm_weight is FP32 contiguous [2, 1, D]; scales FP32 contiguous [H].
 *   - Pointers are device pointers; `stream` is a cudaStream_t (NULL = legacy
 *     default stream). Every call is asynchronous on `stream`.
 *   - The library never allocates or frees device memory and never writes an
 *     input. Callers own every buffer, including backward workspace.
 *   - Every entry point returns an int status (FLASH_PROLOGUE_OK = 0); the
 *     message for a status comes from flash_prologue_status_string().
 *   - dtype codes: 0 = bfloat16, 1 = float16, 2 = float32.
 */
#ifndef FLASH_PROLOGUE_H_
#define FLASH_PROLOGUE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FLASH_PROLOGUE_API __attribute__((visibility("default")))
#else
#define FLASH_PROLOGUE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum flash_prologue_status {
  FLASH_PROLOGUE_OK = 0,
  FLASH_PROLOGUE_ERR_INVALID_ARGUMENT = 1, /* bad size, null pointer, bad eps */
  FLASH_PROLOGUE_ERR_UNSUPPORTED = 2,      /* head_dim / dtype not compiled   */
  FLASH_PROLOGUE_ERR_CHANNEL_STRIDE = 3,   /* d stride != 1                   */
  FLASH_PROLOGUE_ERR_EXPANDED = 4,         /* stride 0 on a dim of size > 1    */
  FLASH_PROLOGUE_ERR_WORKSPACE = 5,        /* workspace missing or too small   */
  FLASH_PROLOGUE_ERR_CUDA = 6,             /* launch or runtime error          */
  FLASH_PROLOGUE_ERR_ALIGNMENT = 7,        /* pointer alignment the path needs */
  FLASH_PROLOGUE_ERR_SCRATCH_LIMIT = 8     /* problem too large for the static scratch */
};

enum flash_prologue_dtype {
  FLASH_PROLOGUE_BF16 = 0,
  FLASH_PROLOGUE_FP16 = 1,
  FLASH_PROLOGUE_FP32 = 2
};

/* Human-readable text for a status code (static storage, never NULL). */
FLASH_PROLOGUE_API const char* flash_prologue_status_string(int status);

/* Library ABI version (major * 100 + minor). */
FLASH_PROLOGUE_API int flash_prologue_version(void);

/*
 * Forward prologue.
 * Replaces the device call of flash_prologue::qknorm_rope_scale_cute
 * (flash_attn_prologue/fused_epilogue.py:702-815, launch at :794) and its
 * kernel FusedEpilogueCute.kernel (fused_epilogue.py:245-576).
 * q_out/k_out may use any strides with d stride 1 (the Python layer passes the
 * reference's compact-by-permutation strides, fused_epilogue.py:688-698).
 * Supported: D in {32, 64, 128, 256}; dtype BF16, FP16, FP32; any eps > 0.
 * B*H*N == 0 returns FLASH_PROLOGUE_OK without a launch.
 */
FLASH_PROLOGUE_API int flash_prologue_fwd(const void* q, const int64_t q_strides[4],
                       const void* k, const int64_t k_strides[4],
                       void* q_out, const int64_t q_out_strides[4],
                       void* k_out, const int64_t k_out_strides[4],
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       int64_t B, int64_t H, int64_t N, int64_t D,
                       float eps, int dtype, void* stream);

/*
 * Bytes of device workspace flash_prologue_bwd needs for this problem on the
 * current device (the per-CTA partial sums of d rmsnorm_weight and d scales).
 * No counterpart in the reference, whose backward zeroes its outputs and
 * accumulates with float atomics (fused_epilogue.py:1403-1404, 1149, 1192-1207).
 */
FLASH_PROLOGUE_API int flash_prologue_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D,
                                      int dtype, size_t* bytes);

/*
 * Backward prologue: dq, dk (input dtype), d rmsnorm_weight [2*D] FP32 and
 * d scales [H] FP32, all overwritten (no zeroing needed). The weight/scale
 * gradients are reduced in a fixed order (per-CTA partials in `workspace`,
 * then a fixed-order pass), so results are bit-identical run to run on the
 * same GPU model.
 * Replaces flash_prologue::qknorm_rope_scale_cute_backward
 * (fused_epilogue.py:1304-1423, launch at :1411) and
 * FusedEpilogueBackwardCute.kernel (fused_epilogue.py:907-1207).
 * Unlike the reference it reads strided q/k/grad views directly instead of
 * copying them to compact strides first (fused_epilogue.py:1338-1344); the
 * upstream gradients may also broadcast (stride 0) over b, h or n.
 * `workspace` must be 16-byte aligned and at least
 * flash_prologue_bwd_workspace_size() bytes; it needs no initialisation.
 */
FLASH_PROLOGUE_API int flash_prologue_bwd(const void* q, const int64_t q_strides[4],
                       const void* k, const int64_t k_strides[4],
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       const void* grad_q_out, const int64_t gq_strides[4],
                       const void* grad_k_out, const int64_t gk_strides[4],
                       void* grad_q, const int64_t dq_strides[4],
                       void* grad_k, const int64_t dk_strides[4],
                       float* grad_rmsnorm_weight, float* grad_scales,
                       void* workspace, size_t workspace_bytes,
                       int64_t B, int64_t H, int64_t N, int64_t D,
                       float eps, int dtype, void* stream);

/*
 * Inverse-formulation forward: flash_prologue_fwd, plus r = 1/sqrt(mean(x^2)+eps)
 * of every row stored to rms_q / rms_k (FP32, contiguous [B, H, N], 4-byte
 * aligned, both required). Saving r and the outputs lets the backward rebuild
 * the normalised rows from the outputs instead of keeping q and k.
 * Replaces flash_prologue::qknorm_rope_scale_cute_inverse
 * (flash_attn_prologue/fused_epilogue.py:2560-2653) and its kernel
 * (fused_epilogue.py:1663-1992), which stores the same statistic
 * (fused_epilogue.py:1916-1917) but fixes eps at 1e-5; this entry point uses `eps`.
 */
FLASH_PROLOGUE_API int flash_prologue_inverse_fwd(const void* q, const int64_t q_strides[4],
                       const void* k, const int64_t k_strides[4],
                       void* q_out, const int64_t q_out_strides[4],
                       void* k_out, const int64_t k_out_strides[4],
                       float* rms_q, float* rms_k,
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       int64_t B, int64_t H, int64_t N, int64_t D,
                       float eps, int dtype, void* stream);

/*
 * Inverse-formulation backward: the results of flash_prologue_bwd computed
 * from the forward OUTPUTS q_out / k_out and the saved r (rms_q / rms_k, FP32
 * contiguous [B, H, N]) instead of q / k. Per row the normalised values are
 * rebuilt as n = R^T(out / exp(scale)) / w (R = the RoPE rotation; the Q scale
 * only on Q), then dq/dk, d rmsnorm_weight and d scales follow as in the
 * backward, with the same fixed-order reduction. Because the outputs were
 * rounded to the activation dtype, the gradients differ from
 * flash_prologue_bwd's by that rounding. `eps` is validated but unused (r is
 * given); `workspace` as for flash_prologue_bwd, whose workspace size also
 * covers this call.
 * Replaces flash_prologue::qknorm_rope_scale_cute_inverse_backward
 * (fused_epilogue.py:2671-2772) and its kernel (fused_epilogue.py:2067-2358),
 * with the reference's float atomics replaced by the fixed-order reduction.
 */
FLASH_PROLOGUE_API int flash_prologue_inverse_bwd(const void* q_out, const int64_t q_out_strides[4],
                       const void* k_out, const int64_t k_out_strides[4],
                       const float* rms_q, const float* rms_k,
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       const void* grad_q_out, const int64_t gq_strides[4],
                       const void* grad_k_out, const int64_t gk_strides[4],
                       void* grad_q, const int64_t dq_strides[4],
                       void* grad_k, const int64_t dk_strides[4],
                       float* grad_rmsnorm_weight, float* grad_scales,
                       void* workspace, size_t workspace_bytes,
                       int64_t B, int64_t H, int64_t N, int64_t D,
                       float eps, int dtype, void* stream);

/*
 * Fused QKV projection GEMM with the prologue in its epilogue (tcgen05 tensor
 * cores, TMEM accumulators, TMA-fed). x: [M, K] BF16 row-major (M = B * S
 * tokens); w: [3*H*D, K] BF16 row-major (nn.Linear layout, rows Q | K | V
 * heads). Computes P = x * w^T, rounds P to BF16, and writes q_out, k_out,
 * v_out as contiguous [B, H, S, D] BF16. With apply_prologue != 0, Q and K get
 * RMSNorm (rmsnorm_weight [2,1,D]), split-half RoPE (sin/cos FP32 indexed
 * [b, s, j] through sin_strides/cos_strides with j stride 1) and Q is
 * multiplied by exp(scales[h]); q_proj/k_proj (optional, may be NULL) receive
 * the BF16 projections before the prologue. With apply_prologue == 0 the
 * prologue arguments may be NULL and Q/K are the plain projections.
 * Requirements: D in {64, 128}; K % 64 == 0; (H*D) % 256 == 0; M % S == 0;
 * x, w and outputs 16-byte aligned.
 * Replaces flash_prologue::fused_qkv (flash_attn_prologue/fused_qkv.py:596-662)
 * and flash_prologue::fused_qkv_epilogue (fused_qkv.py:698-878: GEMM launch,
 * two copies and an in-place prologue launch), one kernel for both.
 */
FLASH_PROLOGUE_API int flash_prologue_qkv_gemm_fwd(const void* x, const void* w,
                       int64_t M, int64_t K, int64_t H, int64_t D, int64_t S,
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       void* q_out, void* k_out, void* v_out,
                       void* q_proj, void* k_proj,
                       float eps, int apply_prologue, void* stream);

/*
 * Backward of the QKV projection P = x * w^T with P split into heads
 * (s = q, k, v): grad_x[b, n, :] = sum_{s,h,d} grad_s[b,h,n,d] * w[(s*H+h)*D+d, :].
 * grad_q/grad_k/grad_v are BF16 [B, H, N, D] views given by element strides
 * (b, h, n, d) with d stride 1 and the others multiples of 8 (a packed
 * [B, N, 3, H, D] gradient is three such views); w: [3*H*D, hidden] and
 * grad_x: [B, N, hidden], both contiguous BF16. tcgen05 GEMM on 2-CTA
 * clusters reading the gradients in place through TMA (no gather of dP).
 * Requirements: D in {64, 128}; (H*D) % 256 == 0; hidden % 64 == 0; 16-byte
 * aligned pointers. Replaces matmul_bwd_dx_cute (flash_attn_prologue/
 * gemm_bwd.py:1171-1235) and the dX half of fused_qkv_backward
 * (gemm_bwd.py:1440-1552).
 */
FLASH_PROLOGUE_API int flash_prologue_qkv_bwd_dx(const void* grad_q, const int64_t gq_strides[4],
                       const void* grad_k, const int64_t gk_strides[4],
                       const void* grad_v, const int64_t gv_strides[4],
                       const void* w, void* grad_x,
                       int64_t B, int64_t H, int64_t N, int64_t D, int64_t hidden,
                       void* stream);

/*
 * Workspace (FP32 split-reduction partials) flash_prologue_qkv_bwd_dw needs on
 * the current device for these sizes; 0 when the sum is empty.
 */
FLASH_PROLOGUE_API int flash_prologue_qkv_bwd_dw_workspace_size(int64_t B, int64_t H, int64_t N,
                       int64_t D, int64_t hidden, size_t* bytes);

/*
 * grad_w[(s*H+h)*D+d, :] = sum_{b,n} grad_s[b,h,n,d] * x[b, n, :] (accumulate
 * == 0), or added to grad_w (accumulate != 0: the FP32 sum plus the old BF16
 * value, rounded once). Gradient views as for flash_prologue_qkv_bwd_dx; x:
 * [B, N, hidden] and grad_w: [3*H*D, hidden], contiguous BF16. The token sum
 * runs as a tcgen05 GEMM in up to 8 chunks written as FP32 partials to the
 * workspace and added in chunk order, so results are identical run to run.
 * Replaces matmul_bwd_dw_cute / matmul_bwd_dw_accumulate_cute
 * (gemm_bwd.py:1246-1421) and the dW half of fused_qkv_backward.
 */
FLASH_PROLOGUE_API int flash_prologue_qkv_bwd_dw(const void* grad_q, const int64_t gq_strides[4],
                       const void* grad_k, const int64_t gk_strides[4],
                       const void* grad_v, const int64_t gv_strides[4],
                       const void* x, void* grad_w, int accumulate,
                       void* workspace, size_t workspace_bytes,
                       int64_t B, int64_t H, int64_t N, int64_t D, int64_t hidden,
                       void* stream);

/*
 * Strided row copy: dst[i0,i1,i2,:] = src[i0,i1,i2,:] for dims[0..2] outer
 * indices (i2 fastest) and rows of row_bytes contiguous bytes, with byte
 * strides src_strides / dst_strides. row_bytes, both base pointers and the
 * strides of dimensions of extent > 1 must be multiples of 16. Moves the V
 * slot of a fused QKV tensor or of its gradient (the reference does these
 * with torch copies: epilogue_kernel.py:222-243, fused_epilogue.py:1399-1402).
 */
FLASH_PROLOGUE_API int flash_prologue_copy_rows(const void* src, const int64_t src_strides[3],
                       void* dst, const int64_t dst_strides[3], const int64_t dims[3],
                       int64_t row_bytes, void* stream);

/*
 * Mainloop of flash_prologue_qkv_gemm_fwd (process-wide, not thread-safe; for
 * tests and tuning). 0 (default): CTA pairs -- 2-CTA clusters running
 * tcgen05.mma.cta_group::2 on 256 x 256 tiles, each CTA loading half of the
 * operands (the single-CTA mainloop is used instead where the device cannot
 * co-schedule 2-CTA clusters); 1: one CTA per SM on 128 x 256 tiles. Both
 * give identical results.
 * No counterpart in the reference (whose GEMM is a CuTe-DSL sm_120a kernel,
 * fused_qkv.py:25, 53-594).
 */
FLASH_PROLOGUE_API int flash_prologue_set_gemm_variant(int variant);

/*
 * Backward prologue that allocates nothing: the same computation and results
 * as flash_prologue_bwd, without the `workspace` arguments. For callers that
 * cannot allocate device memory per call (runtimes that plan all device memory
 * up front, host-language bindings without a device allocator, code running
 * while another framework's pool holds the device heap). Its scratch is a
 * static 1 MiB array in the library's device memory, held by every GPU that
 * loads the library until exit. The first call on a device looks up that
 * array's address with the device current: make it before any stream capture.
 * All calls on a device share the array, so calls that overlap on the GPU race
 * and must be serialised; nothing in it needs clearing between calls.
 * Problems that need more than 1 MiB of scratch (see
 * flash_prologue_bwd_workspace_size) return FLASH_PROLOGUE_ERR_SCRATCH_LIMIT.
 * No counterpart in the reference, whose backward allocates its outputs and
 * zeroed accumulators through PyTorch (fused_epilogue.py:1399-1404).
 */
FLASH_PROLOGUE_API int flash_prologue_bwd_noalloc(const void* q, const int64_t q_strides[4],
                       const void* k, const int64_t k_strides[4],
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       const void* grad_q_out, const int64_t gq_strides[4],
                       const void* grad_k_out, const int64_t gk_strides[4],
                       void* grad_q, const int64_t dq_strides[4],
                       void* grad_k, const int64_t dk_strides[4],
                       float* grad_rmsnorm_weight, float* grad_scales,
                       int64_t B, int64_t H, int64_t N, int64_t D,
                       float eps, int dtype, void* stream);

/*
 * Kernel path selection (process-wide, not thread-safe; for tests and tuning).
 * mode 0 (default): the TMA pipelined kernels whenever the views
 * allow them (16-byte aligned, rows contiguous along the inner row dim, positive
 * 16-byte-multiple outer strides, sin/cos rows contiguous, a tensor map the
 * driver accepts), else the register-path kernels, with the outputs of the
 * pipelined kernels leaving through TMA tensor stores where that measured
 * faster (D = 64 backward, regular or inverse; the D = 64 forward that does
 * not save r, for long runs per CTA) and through the lanes' 16-byte stores
 * otherwise; mode 1: register path
 * only; mode 2: pipelined kernels with TMA-stored outputs wherever the output
 * views allow; mode 3: pipelined kernels with lane stores. Every mode computes
 * bit-identical results.
 * No counterpart in the reference (which has a single kernel per op).
 */
FLASH_PROLOGUE_API int flash_prologue_set_path(int mode);

/*
 * Reads the device error word of the pipelined kernels (0 = none; 1 = a
 * bounded barrier wait gave up, which means the results of that launch are
 * invalid). Synchronous (copies from the device); clears the word if `reset`.
 * No counterpart in the reference (which has no device-side waits).
 */
FLASH_PROLOGUE_API int flash_prologue_device_error(int* value, int reset);

/*
 * Self-test of failure detection: launches one thread that waits, bounded, on
 * an mbarrier that nothing arrives at. After `tries` polls (1 .. 2^22, each
 * suspended up to ~1 us) it gives up and records the timeout in the device
 * error word exactly as a stalled pipelined kernel would, then returns: the
 * context stays usable and flash_prologue_device_error() reports 1. Nothing
 * faults, traps or hangs. No counterpart in the reference.
 */
FLASH_PROLOGUE_API int flash_prologue_selftest_wait_timeout(uint32_t tries, void* stream);

/*
 * ---------------------------------------------------------------------------
 * Data-parallel backward over peer memory (NVLink / NVSwitch). The reference
 * has no distributed code; these entry points make the one collective of the
 * data-parallel step -- the sum over ranks of d rmsnorm_weight and d scales --
 * part of the backward's own finalize kernel instead of a separate library
 * collective. One process per GPU, all GPUs of one node.
 *
 * A peer group is one small exchange buffer and one flag array per rank,
 * allocated by each rank (from its own allocator, zero-filled) and mapped into
 * every other rank's address space with the IPC calls below. The descriptor
 * lists every rank's buffers as mapped in the calling process (its own at
 * index `rank`).
 */
#define FLASH_PROLOGUE_MAX_PEERS 8

typedef struct flash_prologue_peers {
  int32_t world;      /* ranks in the group, 1 .. FLASH_PROLOGUE_MAX_PEERS          */
  int32_t rank;       /* the calling rank                                         */
  int32_t max_cols;   /* floats per exchange row: >= 2 * D + H, a multiple of 32  */
  int32_t wait_ms;    /* bound on each wait for a peer, ms; 0 = 2000, at most 60000 */
  float* data[FLASH_PROLOGUE_MAX_PEERS];      /* [2][world][max_cols] FP32 per rank */
  uint32_t* flags[FLASH_PROLOGUE_MAX_PEERS];  /* [2][world][max_cols / 32] per rank */
} flash_prologue_peers;

/* Bytes of one rank's exchange buffer and flag array for a group shape. */
FLASH_PROLOGUE_API int flash_prologue_peer_buffer_bytes(int32_t world, int32_t max_cols,
                                                        size_t* data_bytes, size_t* flag_bytes);

/*
 * IPC mapping of device memory between the processes of one node:
 * `handle` (64 bytes) names the allocation holding `dev_ptr`, `offset` is
 * dev_ptr's offset in it; open maps a peer's handle and returns its pointer
 * plus offset; close unmaps what open returned. The caller's allocation must
 * stay alive while any peer has it open.
 */
FLASH_PROLOGUE_API int flash_prologue_ipc_handle(const void* dev_ptr, void* handle, int64_t* offset);
FLASH_PROLOGUE_API int flash_prologue_ipc_open(const void* handle, int64_t offset, void** dev_ptr);
FLASH_PROLOGUE_API int flash_prologue_ipc_close(void* dev_ptr, int64_t offset);

/*
 * flash_prologue_bwd whose d rmsnorm_weight / d scales come out summed over
 * the ranks of `peers`: the finalize kernel adds the per-CTA partials in a
 * fixed order, writes the rank's sum into every rank's exchange buffer over
 * NVLink, sets its flags there, waits (bounded) for every rank's flags in its
 * own buffer and adds the ranks' sums in rank order -- the same bits on every
 * rank and run to run. `epoch` must be the same on every rank and grow by one
 * per call (start at 1); calls alternate between two halves of the buffers, so
 * a rank may run one call ahead of the slowest. Every rank must make the same
 * calls in the same order. A wait that runs out (a rank that did not arrive)
 * records the device error word and writes NaN gradients; nothing hangs. The
 * ranks must be on different GPUs: two ranks on one GPU would be separate
 * kernels waiting on each other, which the GPU need not run side by side.
 */
FLASH_PROLOGUE_API int flash_prologue_bwd_dp(const void* q, const int64_t q_strides[4],
                       const void* k, const int64_t k_strides[4],
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       const void* grad_q_out, const int64_t gq_strides[4],
                       const void* grad_k_out, const int64_t gk_strides[4],
                       void* grad_q, const int64_t dq_strides[4],
                       void* grad_k, const int64_t dk_strides[4],
                       float* grad_rmsnorm_weight, float* grad_scales,
                       void* workspace, size_t workspace_bytes,
                       int64_t B, int64_t H, int64_t N, int64_t D,
                       float eps, int dtype, const flash_prologue_peers* peers,
                       uint32_t epoch, void* stream);

/*
 * flash_prologue_inverse_bwd with the same group reduction of d rmsnorm_weight
 * and d scales (same epoch sequence as flash_prologue_bwd_dp: one counter per
 * group, whichever of the two a call uses).
 */
FLASH_PROLOGUE_API int flash_prologue_inverse_bwd_dp(const void* q_out, const int64_t q_out_strides[4],
                       const void* k_out, const int64_t k_out_strides[4],
                       const float* rms_q, const float* rms_k,
                       const float* rmsnorm_weight, const float* scales,
                       const float* sin, const int64_t sin_strides[3],
                       const float* cos, const int64_t cos_strides[3],
                       const void* grad_q_out, const int64_t gq_strides[4],
                       const void* grad_k_out, const int64_t gk_strides[4],
                       void* grad_q, const int64_t dq_strides[4],
                       void* grad_k, const int64_t dk_strides[4],
                       float* grad_rmsnorm_weight, float* grad_scales,
                       void* workspace, size_t workspace_bytes,
                       int64_t B, int64_t H, int64_t N, int64_t D,
                       float eps, int dtype, const flash_prologue_peers* peers,
                       uint32_t epoch, void* stream);

/*
 * Test form of the group reduction: every rank of `peers` emulated by one
 * cooperative launch on the current GPU (all buffers local). partials[r]:
 * rank r's [G, C] per-CTA partials; dw[r] / ds[r]: its outputs. For tests on
 * one GPU of the protocol flash_prologue_bwd_dp runs across GPUs.
 */
FLASH_PROLOGUE_API int flash_prologue_peer_reduce_emulated(const float* const* partials, int64_t G,
                       int32_t C, int32_t two_d, float* const* dw, float* const* ds,
                       const flash_prologue_peers* peers, uint32_t epoch, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* FLASH_PROLOGUE_H_ */
