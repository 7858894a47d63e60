"""Fused QKV projection with the prologue in the GEMM epilogue (tcgen05/TMEM, sm_100a).

Custom ops under the reference's names (flash_attn_prologue/fused_qkv.py):

* ``flash_prologue::fused_qkv(x, weight) -> (q, k, v)``: the projection
  ``x @ weight.T`` split into per-head ``[B, H, N, D]`` BF16 tensors
  (reference: fused_qkv.py:596-662);
* ``flash_prologue::fused_qkv_epilogue(x, weight, rmsnorm_weight, scales, sin, cos)
  -> (q, k, v, q_proj, k_proj)``: the same projection with RMSNorm + RoPE + Q
  scale applied to Q and K inside the GEMM epilogue, plus the pre-prologue
  BF16 projections the backward uses (reference: fused_qkv.py:698-878, which
  runs a GEMM, two copies and a separate prologue launch);
* ``flash_prologue::fused_qkv_epilogue_ckp(...) -> (q, k, v)``: the recompute
  variant that keeps no projections (reference: fused_qkv.py:880-1053);
* the projection backward ops ``fused_qkv_backward``, ``matmul_bwd_dx_cute``,
  ``matmul_bwd_dw_cute``, ``matmul_bwd_dw_accumulate_cute`` and the Python
  ``matmul_bwd_dx`` / ``matmul_bwd_dw`` (reference: gemm_bwd.py:1171-1566),
  as two tcgen05 GEMM kernels (csrc/qkv_gemm_bwd.cu) that read the per-head
  gradients in place.

``weight`` is the nn.Linear weight ``[3*H*D, hidden]`` with rows Q heads | K
heads | V heads; D is taken from ``rmsnorm_weight`` (the reference hard-codes
64, fused_qkv.py:606-607); H = weight.shape[0] // (3 * D). The projection is
rounded to BF16 before the prologue, as a BF16 linear layer followed by the
prologue would do. Backward: the prologue backward kernel on the saved
(or recomputed) projections, then dX = dP @ W and dW = dP^T @ X by the
backward GEMM kernels reading dq, dk, dv in place as the head blocks of dP.
"""
from typing import Optional, Tuple

import torch

from . import _lib
from .fused_epilogue import _DeviceGuard, _ensure_4d, _table, backward_into

BN_TILE = 256


def _dims(x: torch.Tensor, weight: torch.Tensor, head_dim: int):
    if x.ndim != 3 or weight.ndim != 2 or x.shape[2] != weight.shape[1]:
        raise ValueError("x must be [B, N, hidden] and weight [3*H*D, hidden]")
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("the fused QKV GEMM takes BF16 x and weight")
    if head_dim not in (64, 128) or weight.shape[0] % (3 * head_dim):
        raise ValueError("weight rows must be 3 * H * D with D in (64, 128)")
    B, N, hidden = (int(s) for s in x.shape)
    H = int(weight.shape[0]) // (3 * head_dim)
    if (H * head_dim) % BN_TILE or hidden % 64:
        raise ValueError("H * D must be a multiple of 256 and hidden a multiple of 64")
    return B, N, hidden, H


def _launch(x, weight, head_dim, outs, raws, rmsnorm_weight=None, scales=None, sin=None, cos=None,
            eps=1e-5):
    B, N, hidden, H = _dims(x, weight, head_dim)
    if B * N == 0:
        return
    x2 = x.reshape(B * N, hidden)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    w2 = weight if weight.is_contiguous() else weight.contiguous()
    lib = _lib.load()
    apply = rmsnorm_weight is not None
    if apply:
        sin4, sin_str = _table(sin, B, N, head_dim // 2)
        cos4, cos_str = _table(cos, B, N, head_dim // 2)
        if sin_str[2] != 1 or sin4.data_ptr() % 16 or sin_str[1] % 4 or sin_str[0] % 4:
            sin4 = sin4.contiguous()
            sin_str = (sin4.stride(0) if sin4.shape[0] > 1 else 0,
                       sin4.stride(2) if sin4.shape[2] > 1 else 0, 1)
        if cos_str[2] != 1 or cos4.data_ptr() % 16 or cos_str[1] % 4 or cos_str[0] % 4:
            cos4 = cos4.contiguous()
            cos_str = (cos4.stride(0) if cos4.shape[0] > 1 else 0,
                       cos4.stride(2) if cos4.shape[2] > 1 else 0, 1)
        w = rmsnorm_weight.contiguous()
        s = scales.contiguous()
        tab = (_lib.ptr(w), _lib.ptr(s), _lib.ptr(sin4), _lib.strides3(sin_str), _lib.ptr(cos4),
               _lib.strides3(cos_str))
    else:
        null = _lib.ctypes.c_void_p(0)
        tab = (null, null, null, None, null, None)
    with _DeviceGuard(x.device):
        status = lib.flash_prologue_qkv_gemm_fwd(
            _lib.ptr(x2), _lib.ptr(w2), B * N, hidden, H, head_dim, N, *tab,
            _lib.ptr(outs[0]), _lib.ptr(outs[1]), _lib.ptr(outs[2]),
            _lib.ptr(raws[0]) if raws[0] is not None else None,
            _lib.ptr(raws[1]) if raws[1] is not None else None,
            float(eps), 1 if apply else 0, _lib.stream_of(x.device))
    _lib.check(status, "flash_prologue_qkv_gemm_fwd")


def _empty_bhnd(x, H, head_dim):
    B, N = x.shape[0], x.shape[1]
    return torch.empty((B, H, N, head_dim), dtype=torch.bfloat16, device=x.device)


# The GEMM-only op has no rmsnorm_weight to read D from; like the reference
# (fused_qkv.py:606-607) it splits the projection into heads of 64.
GEMM_ONLY_HEAD_DIM = 64


@torch.library.custom_op("flash_prologue::fused_qkv", mutates_args=())
def fused_qkv_op(x: torch.Tensor, weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    head_dim = GEMM_ONLY_HEAD_DIM
    _, _, _, H = _dims(x, weight, head_dim)
    outs = [_empty_bhnd(x, H, head_dim) for _ in range(3)]
    _launch(x, weight, head_dim, outs, (None, None))
    return outs[0], outs[1], outs[2]


@fused_qkv_op.register_fake
def _fused_qkv_fake(x, weight):
    head_dim = GEMM_ONLY_HEAD_DIM
    H = weight.shape[0] // (3 * head_dim)
    return tuple(torch.empty((x.shape[0], H, x.shape[1], head_dim), dtype=x.dtype, device=x.device)
                 for _ in range(3))


def _check_grads_qkv(grad_q, grad_k, grad_v):
    if grad_q.ndim != 4 or grad_k.shape != grad_q.shape or grad_v.shape != grad_q.shape:
        raise ValueError("grad_q/grad_k/grad_v must be matching [B, H, N, D] tensors")


def _tma_view(g: torch.Tensor) -> torch.Tensor:
    """g itself when the backward GEMMs can read it in place (BF16, d contiguous,
    16-byte aligned base and row strides), else a contiguous copy."""
    if g.dtype != torch.bfloat16:
        raise ValueError("the projection backward takes BF16 gradients")
    st = g.stride()
    ok = (st[3] == 1 and g.data_ptr() % 16 == 0 and
          all(st[i] % 8 == 0 and st[i] > 0 for i in range(3) if g.shape[i] > 1))
    return g if ok else g.contiguous()


def _check_bwd_shapes(B, H, N, D, hidden, device):
    if device.type != "cuda":
        raise ValueError("the projection backward GEMMs run on CUDA devices only")
    if D not in (64, 128) or (H * D) % BN_TILE or hidden % 64:
        raise ValueError("the projection backward needs D in (64, 128), H * D a multiple of 256 "
                         "and hidden a multiple of 64")


def _bwd_dx(dq, dk, dv, weight):
    """dX [B, N, hidden] = dP @ weight, dP read from the [B, H, N, D] gradients in place."""
    B, H, N, D = dq.shape
    hidden = int(weight.shape[1])
    _check_bwd_shapes(B, H, N, D, hidden, dq.device)
    if weight.dtype != torch.bfloat16 or tuple(weight.shape) != (3 * H * D, hidden):
        raise ValueError("weight must be BF16 [3*H*D, hidden]")
    w = weight.contiguous()
    views = [_tma_view(g) for g in (dq, dk, dv)]
    grad_x = torch.empty((B, N, hidden), dtype=torch.bfloat16, device=dq.device)
    with _DeviceGuard(dq.device):
        status = _lib.load().flash_prologue_qkv_bwd_dx(
            _lib.ptr(views[0]), _lib.strides4(views[0]), _lib.ptr(views[1]), _lib.strides4(views[1]),
            _lib.ptr(views[2]), _lib.strides4(views[2]), _lib.ptr(w), _lib.ptr(grad_x),
            B, H, N, D, hidden, _lib.stream_of(dq.device))
    _lib.check(status, "flash_prologue_qkv_bwd_dx")
    return grad_x


def _bwd_dw(dq, dk, dv, x, out=None):
    """dW [3*H*D, hidden] = dP^T @ x (or added to ``out``), dP read in place."""
    B, H, N, D = dq.shape
    hidden = int(x.shape[-1])
    _check_bwd_shapes(B, H, N, D, hidden, dq.device)
    if x.dtype != torch.bfloat16 or x.numel() != B * N * hidden:
        raise ValueError("x must be BF16 [B, N, hidden]")
    x3 = x.reshape(B, N, hidden).contiguous()
    views = [_tma_view(g) for g in (dq, dk, dv)]
    grad_w = out if out is not None else torch.empty((3 * H * D, hidden), dtype=torch.bfloat16,
                                                      device=dq.device)
    if out is not None and (out.dtype != torch.bfloat16 or tuple(out.shape) != (3 * H * D, hidden)
                            or not out.is_contiguous()):
        raise ValueError("out must be a contiguous BF16 [3*H*D, hidden] tensor")
    lib = _lib.load()
    with _DeviceGuard(dq.device):
        nbytes = _lib.ctypes.c_size_t(0)
        _lib.check(lib.flash_prologue_qkv_bwd_dw_workspace_size(B, H, N, D, hidden,
                                                                _lib.ctypes.byref(nbytes)),
                   "flash_prologue_qkv_bwd_dw_workspace_size")
        ws = torch.empty(max(int(nbytes.value), 16), dtype=torch.uint8, device=dq.device)
        status = lib.flash_prologue_qkv_bwd_dw(
            _lib.ptr(views[0]), _lib.strides4(views[0]), _lib.ptr(views[1]), _lib.strides4(views[1]),
            _lib.ptr(views[2]), _lib.strides4(views[2]), _lib.ptr(x3), _lib.ptr(grad_w),
            1 if out is not None else 0, _lib.ptr(ws), int(nbytes.value), B, H, N, D, hidden,
            _lib.stream_of(dq.device))
    _lib.check(status, "flash_prologue_qkv_bwd_dw")
    return grad_w


@torch.library.custom_op("flash_prologue::matmul_bwd_dx_cute", mutates_args=())
def matmul_bwd_dx(grad_q: torch.Tensor, grad_k: torch.Tensor, grad_v: torch.Tensor,
                  weight: torch.Tensor) -> torch.Tensor:
    """dX = dP @ weight as [B*N, hidden] (reference: gemm_bwd.py:1171-1235)."""
    _check_grads_qkv(grad_q, grad_k, grad_v)
    B, H, N, D = grad_q.shape
    if grad_q.numel() == 0 or weight.numel() == 0:
        return torch.zeros((B * N, weight.shape[1]), dtype=grad_q.dtype, device=grad_q.device)
    return _bwd_dx(grad_q, grad_k, grad_v, weight).view(B * N, weight.shape[1])


@matmul_bwd_dx.register_fake
def _matmul_bwd_dx_fake(grad_q, grad_k, grad_v, weight):
    B, H, N, D = grad_q.shape
    return torch.empty((B * N, weight.shape[1]), dtype=grad_q.dtype, device=grad_q.device)


@torch.library.custom_op("flash_prologue::matmul_bwd_dw_cute", mutates_args=())
def _matmul_bwd_dw_op(grad_q: torch.Tensor, grad_k: torch.Tensor, grad_v: torch.Tensor,
                      x: torch.Tensor) -> torch.Tensor:
    """dW = dP^T @ X as [3*H*D, hidden] (reference: gemm_bwd.py:1246-1330)."""
    _check_grads_qkv(grad_q, grad_k, grad_v)
    B, H, N, D = grad_q.shape
    hidden = x.shape[-1]
    if grad_q.numel() == 0 or x.numel() == 0:
        return torch.zeros((3 * H * D, hidden), dtype=grad_q.dtype, device=grad_q.device)
    return _bwd_dw(grad_q, grad_k, grad_v, x)


@_matmul_bwd_dw_op.register_fake
def _matmul_bwd_dw_fake(grad_q, grad_k, grad_v, x):
    B, H, N, D = grad_q.shape
    return torch.empty((3 * H * D, x.shape[-1]), dtype=grad_q.dtype, device=grad_q.device)


@torch.library.custom_op("flash_prologue::matmul_bwd_dw_accumulate_cute", mutates_args={"out"})
def _matmul_bwd_dw_accumulate_op(grad_q: torch.Tensor, grad_k: torch.Tensor, grad_v: torch.Tensor,
                                 x: torch.Tensor, out: torch.Tensor) -> None:
    """out += dP^T @ X in place (reference: gemm_bwd.py:1341-1421)."""
    _check_grads_qkv(grad_q, grad_k, grad_v)
    if grad_q.numel() == 0 or x.numel() == 0:
        return
    _bwd_dw(grad_q, grad_k, grad_v, x, out=out)


@_matmul_bwd_dw_accumulate_op.register_fake
def _matmul_bwd_dw_accumulate_fake(grad_q, grad_k, grad_v, x, out):
    return None


def matmul_bwd_dw(grad_q, grad_k, grad_v, x, out=None):
    """dW = dP^T @ X; with ``out``, accumulated into it (reference: gemm_bwd.py:1427-1438)."""
    if out is None:
        return torch.ops.flash_prologue.matmul_bwd_dw_cute(grad_q, grad_k, grad_v, x)
    torch.ops.flash_prologue.matmul_bwd_dw_accumulate_cute(grad_q, grad_k, grad_v, x, out)
    return out


def _slot_views(dp5):
    """The q, k, v gradient views [B, H, N, D] of a packed [B, N, 3, H, D] dP."""
    return [dp5[:, :, i].permute(0, 2, 1, 3) for i in range(3)]


@torch.library.custom_op("flash_prologue::fused_qkv_backward", mutates_args=())
def fused_qkv_backward(grad_q: torch.Tensor, grad_k: torch.Tensor, grad_v: torch.Tensor,
                       weight: torch.Tensor, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(grad_x [B, N, hidden], grad_weight [3*H*D, hidden]) of P = x @ weight.T split into heads.

    Reference: gemm_bwd.py:1440-1552. Here two tcgen05 GEMM kernels read the
    three gradients in place (no gather of dP). Empty inputs give zeros.
    """
    _check_grads_qkv(grad_q, grad_k, grad_v)
    B, H, N, D = grad_q.shape
    hidden = weight.shape[1]
    if grad_q.numel() == 0 or x.numel() == 0 or weight.numel() == 0:
        return (torch.zeros((B, N, hidden), dtype=grad_q.dtype, device=grad_q.device),
                torch.zeros((3 * H * D, hidden), dtype=grad_q.dtype, device=grad_q.device))
    return _bwd_dx(grad_q, grad_k, grad_v, weight), _bwd_dw(grad_q, grad_k, grad_v, x)


@fused_qkv_backward.register_fake
def _fused_qkv_backward_fake(grad_q, grad_k, grad_v, weight, x):
    B, H, N, D = grad_q.shape
    hidden = weight.shape[1]
    return (torch.empty((B, N, hidden), dtype=grad_q.dtype, device=grad_q.device),
            torch.empty((3 * H * D, hidden), dtype=grad_q.dtype, device=grad_q.device))


def _linear_backward(dq, dk, dv, weight, x):
    return fused_qkv_backward(dq, dk, dv, weight, x)


def _fused_qkv_setup(ctx, inputs, output):
    x, weight = inputs
    ctx.save_for_backward(x, weight)


def _fused_qkv_backward(ctx, gq, gk, gv):
    x, weight = ctx.saved_tensors
    return _linear_backward(gq, gk, gv, weight, x)


torch.library.register_autograd("flash_prologue::fused_qkv", _fused_qkv_backward,
                                setup_context=_fused_qkv_setup)


@torch.library.custom_op("flash_prologue::fused_qkv_epilogue", mutates_args=())
def fused_qkv_epilogue_op(
    x: torch.Tensor,
    weight: torch.Tensor,
    rmsnorm_weight: torch.Tensor,
    scales: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    # eps: a trailing optional argument beyond the reference's schema (which
    # fixes 1e-5); callers of the reference's six-argument form are unaffected.
    head_dim, H = _check_prologue_params(x, weight, rmsnorm_weight, scales, sin, cos)
    _check_eps(eps)
    outs = [_empty_bhnd(x, H, head_dim) for _ in range(3)]
    raws = [_empty_bhnd(x, H, head_dim) for _ in range(2)]
    _launch(x, weight, head_dim, outs, raws, rmsnorm_weight, scales, sin, cos, eps)
    return outs[0], outs[1], outs[2], raws[0], raws[1]


@fused_qkv_epilogue_op.register_fake
def _fused_qkv_epilogue_fake(x, weight, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    head_dim = rmsnorm_weight.shape[-1]
    H = weight.shape[0] // (3 * head_dim)
    return tuple(torch.empty((x.shape[0], H, x.shape[1], head_dim), dtype=x.dtype, device=x.device)
                 for _ in range(5))


def _prologue_and_linear_backward(x, weight, rmsnorm_weight, scales, sin, cos, q_proj, k_proj,
                                  grad_q, grad_k, grad_v, eps=1e-5):
    """(grad_x, grad_w, dw, ds) of the fused projection + prologue.

    The prologue backward kernel writes dq and dk into a [B, N, 2, H, D]
    buffer; the backward GEMM kernels then read dq, dk and the upstream dv in
    place as the three head blocks of dP (dX = dP @ W, dW = dP^T @ X).
    """
    B, H, N, D = q_proj.shape
    dqk = torch.empty((B, N, 2, H, D), dtype=q_proj.dtype, device=q_proj.device)
    dq = dqk[:, :, 0].permute(0, 2, 1, 3)
    dk = dqk[:, :, 1].permute(0, 2, 1, 3)
    sin4 = _ensure_4d(sin).expand(B, 1, N, D // 2)
    cos4 = _ensure_4d(cos).expand(B, 1, N, D // 2)
    dw, ds = backward_into(q_proj, k_proj, rmsnorm_weight, scales, sin4, cos4, grad_q, grad_k,
                           dq, dk, eps)
    if B * N == 0:
        return (torch.zeros_like(x), torch.zeros_like(weight), dw, ds)
    dv = torch.zeros_like(q_proj) if grad_v is None else grad_v
    return _bwd_dx(dq, dk, dv, weight), _bwd_dw(dq, dk, dv, x), dw, ds


@torch.library.custom_op("flash_prologue::fused_qkv_epilogue_backward", mutates_args=())
def fused_qkv_epilogue_backward_op(
    x: torch.Tensor, weight: torch.Tensor, rmsnorm_weight: torch.Tensor, scales: torch.Tensor,
    sin: torch.Tensor, cos: torch.Tensor, q_proj: torch.Tensor, k_proj: torch.Tensor,
    grad_q: Optional[torch.Tensor], grad_k: Optional[torch.Tensor], grad_v: Optional[torch.Tensor],
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Backward of fused_qkv_epilogue from its saved BF16 projections (reference: fused_qkv.py:847-867)."""
    return _prologue_and_linear_backward(x, weight, rmsnorm_weight, scales, sin, cos, q_proj, k_proj,
                                         grad_q, grad_k, grad_v, eps)


@fused_qkv_epilogue_backward_op.register_fake
def _fused_qkv_epilogue_backward_fake(x, weight, rmsnorm_weight, scales, sin, cos, q_proj, k_proj,
                                      grad_q, grad_k, grad_v, eps=1e-5):
    D, H = q_proj.shape[-1], q_proj.shape[1]
    return (torch.empty_like(x), torch.empty_like(weight),
            torch.empty((2, 1, D), dtype=torch.float32, device=x.device),
            torch.empty((H, 1, 1), dtype=torch.float32, device=x.device))


def _fused_qkv_epilogue_setup(ctx, inputs, output):
    x, weight, rmsnorm_weight, scales, sin, cos, eps = inputs
    _, _, _, q_proj, k_proj = output
    ctx.save_for_backward(x, weight, rmsnorm_weight, scales, sin, cos, q_proj, k_proj)
    ctx.eps = eps


def _fused_qkv_epilogue_backward(ctx, gq, gk, gv, g_qproj, g_kproj):
    # The saved projections are outputs for the backward only; as in the
    # reference (fused_qkv.py:847-867) gradients arriving on them are ignored.
    x, weight, rmsnorm_weight, scales, sin, cos, q_proj, k_proj = ctx.saved_tensors
    grad_x, grad_w, dw, ds = fused_qkv_epilogue_backward_op(
        x, weight, rmsnorm_weight, scales, sin, cos, q_proj, k_proj, gq, gk, gv, ctx.eps)
    return grad_x, grad_w, dw, ds, None, None, None


torch.library.register_autograd("flash_prologue::fused_qkv_epilogue", _fused_qkv_epilogue_backward,
                                setup_context=_fused_qkv_epilogue_setup)


# ---------------------------------------------------------------------------
# Recompute (checkpoint) composite: the forward keeps no projections; the
# backward recomputes them with the GEMM kernel (reference: fused_qkv.py:880-1053).

def _check_prologue_params(x, weight, rmsnorm_weight, scales, sin, cos):
    head_dim = int(rmsnorm_weight.shape[-1])
    _, _, _, H = _dims(x, weight, head_dim)
    if tuple(rmsnorm_weight.shape) != (2, 1, head_dim) or scales.numel() != H:
        raise ValueError("weight must be [2,1,D], log-scales must be [H,1,1]")
    for t in (rmsnorm_weight, scales, sin, cos):
        if t.dtype != torch.float32:
            raise ValueError("weights, log-scales, and sin/cos must be FP32")
    return head_dim, H


def _check_eps(eps):
    if not (eps > 0.0) or eps == float("inf"):
        raise ValueError("eps must be finite and positive")


@torch.library.custom_op("flash_prologue::fused_qkv_epilogue_ckp", mutates_args=())
def fused_qkv_epilogue_ckp_op(
    x: torch.Tensor, weight: torch.Tensor, rmsnorm_weight: torch.Tensor, scales: torch.Tensor,
    sin: torch.Tensor, cos: torch.Tensor, eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(q, k, v) of fused_qkv_epilogue without storing the pre-prologue projections."""
    head_dim, H = _check_prologue_params(x, weight, rmsnorm_weight, scales, sin, cos)
    _check_eps(eps)
    outs = [_empty_bhnd(x, H, head_dim) for _ in range(3)]
    _launch(x, weight, head_dim, outs, (None, None), rmsnorm_weight, scales, sin, cos, eps)
    return outs[0], outs[1], outs[2]


@fused_qkv_epilogue_ckp_op.register_fake
def _fused_qkv_epilogue_ckp_fake(x, weight, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    head_dim = rmsnorm_weight.shape[-1]
    H = weight.shape[0] // (3 * head_dim)
    return tuple(torch.empty((x.shape[0], H, x.shape[1], head_dim), dtype=x.dtype, device=x.device)
                 for _ in range(3))


@torch.library.custom_op("flash_prologue::fused_qkv_epilogue_ckp_backward", mutates_args=())
def fused_qkv_epilogue_ckp_backward_op(
    x: torch.Tensor, weight: torch.Tensor, rmsnorm_weight: torch.Tensor, scales: torch.Tensor,
    sin: torch.Tensor, cos: torch.Tensor, grad_q: Optional[torch.Tensor],
    grad_k: Optional[torch.Tensor], grad_v: Optional[torch.Tensor], eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Recomputes the BF16 projections (same kernel, bit-identical), then the fused backward."""
    head_dim, H = _check_prologue_params(x, weight, rmsnorm_weight, scales, sin, cos)
    proj = [_empty_bhnd(x, H, head_dim) for _ in range(3)]
    _launch(x, weight, head_dim, proj, (None, None))
    return _prologue_and_linear_backward(x, weight, rmsnorm_weight, scales, sin, cos, proj[0], proj[1],
                                         grad_q, grad_k, grad_v, eps)


@fused_qkv_epilogue_ckp_backward_op.register_fake
def _fused_qkv_epilogue_ckp_backward_fake(x, weight, rmsnorm_weight, scales, sin, cos, grad_q, grad_k,
                                          grad_v, eps=1e-5):
    D = rmsnorm_weight.shape[-1]
    H = weight.shape[0] // (3 * D)
    return (torch.empty_like(x), torch.empty_like(weight),
            torch.empty((2, 1, D), dtype=torch.float32, device=x.device),
            torch.empty((H, 1, 1), dtype=torch.float32, device=x.device))


def _fused_qkv_epilogue_ckp_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs[:6])
    ctx.eps = inputs[6]


def _fused_qkv_epilogue_ckp_backward(ctx, gq, gk, gv):
    grad_x, grad_w, dw, ds = fused_qkv_epilogue_ckp_backward_op(*ctx.saved_tensors, gq, gk, gv, ctx.eps)
    return grad_x, grad_w, dw, ds, None, None, None


torch.library.register_autograd("flash_prologue::fused_qkv_epilogue_ckp", _fused_qkv_epilogue_ckp_backward,
                                setup_context=_fused_qkv_epilogue_ckp_setup)
