"""``flash_prologue::qknorm_rope_scale``: the prologue on a fused ``[B, N, 3*H*D]`` QKV activation.

Same op name, schema and outputs as the reference's
(flash_attn_prologue/epilogue_kernel.py:247-369): ``qkv`` is the QKV
projection ``[B, N, 3*H*D]`` (Q heads | K heads | V heads), and the op returns
``(q, k, v)`` as contiguous ``[B, H, N, D]`` tensors -- Q and K through the
prologue, V copied out. The reference runs its CuTe prologue op on contiguous
copies of the Q and K slices (epilogue_kernel.py:222-243); here the kernels
read the slices of ``qkv`` in place and write the contiguous outputs directly
(V by the library's row copy).
Backward: the prologue backward kernel writes dq and dk straight into the Q/K
slots of one ``[B, N, 3*H*D]`` gradient and dv is copied into its V slot
(the exact gradient of the forward; the reference's backward is an eager
formulation with BF16-rounded intermediates, epilogue_kernel.py:290-362).
CUDA only: the reference's CPU path (an eager restatement) is not part of
this build, and a CPU tensor raises.
"""
from typing import Tuple

import torch

from . import _lib
from .fused_epilogue import (_check_common, _DeviceGuard, _ensure_4d, _table,
                             qknorm_rope_scale_qkv_backward_op)


def _weight3(rmsnorm_weight: torch.Tensor) -> torch.Tensor:
    """[2, D] or [2, 1, D] RMSNorm weight as [2, 1, D] (both accepted, epilogue_kernel.py:194)."""
    return rmsnorm_weight.unsqueeze(1) if rmsnorm_weight.dim() == 2 else rmsnorm_weight


def _split(qkv: torch.Tensor, rmsnorm_weight: torch.Tensor, scales: torch.Tensor):
    if qkv.ndim != 3:
        raise ValueError("qkv must be [B, N, 3*H*D]")
    H = int(scales.shape[0])
    D = int(rmsnorm_weight.shape[-1])
    B, N, total = (int(x) for x in qkv.shape)
    if total != 3 * H * D:
        raise ValueError("qkv's last dimension must be 3 * H * D")
    if qkv.stride(-1) != 1:
        qkv = qkv.contiguous()
    return qkv.view(B, N, 3, H, D) if qkv.is_contiguous() else qkv.reshape(B, N, 3, H, D), B, N, H, D


@torch.library.custom_op("flash_prologue::qknorm_rope_scale", mutates_args=())
def qknorm_rope_scale_op(
    qkv: torch.Tensor,
    rmsnorm_weight: torch.Tensor,
    scales: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    if qkv.device.type != "cuda":
        raise ValueError("flash_prologue::qknorm_rope_scale runs on CUDA devices only")
    rmsnorm_weight = _weight3(rmsnorm_weight)
    qkv5, B, N, H, D = _split(qkv, rmsnorm_weight, scales)
    q4 = qkv5[:, :, 0].permute(0, 2, 1, 3)
    k4 = qkv5[:, :, 1].permute(0, 2, 1, 3)
    sin4 = _ensure_4d(sin)
    cos4 = _ensure_4d(cos)
    _check_common(q4, k4, rmsnorm_weight, scales, sin4, cos4, eps)
    q_out = torch.empty((B, H, N, D), dtype=qkv.dtype, device=qkv.device)
    k_out = torch.empty((B, H, N, D), dtype=qkv.dtype, device=qkv.device)
    v_out = torch.empty((B, H, N, D), dtype=qkv.dtype, device=qkv.device)
    _lib.copy_rows(v_out, qkv5[:, :, 2].permute(0, 2, 1, 3))
    if q4.numel() == 0:
        return q_out, k_out, v_out
    s4, sin_str = _table(sin4, B, N, D // 2)
    c4, cos_str = _table(cos4, B, N, D // 2)
    w = rmsnorm_weight.float().contiguous()
    s = scales.float().contiguous()
    with _DeviceGuard(qkv.device):
        status = _lib.load().flash_prologue_fwd(
            _lib.ptr(q4), _lib.strides4(q4), _lib.ptr(k4), _lib.strides4(k4),
            _lib.ptr(q_out), _lib.strides4(q_out), _lib.ptr(k_out), _lib.strides4(k_out),
            _lib.ptr(w), _lib.ptr(s),
            _lib.ptr(s4), _lib.strides3(sin_str), _lib.ptr(c4), _lib.strides3(cos_str),
            B, H, N, D, float(eps), _lib.DTYPE_CODES[qkv.dtype], _lib.stream_of(qkv.device))
    _lib.check(status, "flash_prologue_fwd")
    return q_out, k_out, v_out


@qknorm_rope_scale_op.register_fake
def _qknorm_rope_scale_fake(qkv, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    B, N, _ = qkv.shape
    H, D = scales.shape[0], rmsnorm_weight.shape[-1]
    return tuple(torch.empty((B, H, N, D), dtype=qkv.dtype, device=qkv.device) for _ in range(3))


def _setup_context(ctx, inputs, output):
    qkv, rmsnorm_weight, scales, sin, cos, eps = inputs
    ctx.save_for_backward(qkv, rmsnorm_weight, scales, sin, cos)
    ctx.eps = eps


def _backward(ctx, grad_q, grad_k, grad_v):
    qkv, rmsnorm_weight, scales, sin, cos = ctx.saved_tensors
    w3 = _weight3(rmsnorm_weight)
    qkv5, B, N, H, D = _split(qkv, w3, scales)
    gv = None if grad_v is None else grad_v.permute(0, 2, 1, 3)
    grad_qkv, dw, ds = qknorm_rope_scale_qkv_backward_op(qkv5, w3, scales, _ensure_4d(sin), _ensure_4d(cos),
                                                         grad_q, grad_k, gv, ctx.eps)
    return (grad_qkv.reshape(B, N, 3 * H * D), dw.reshape(rmsnorm_weight.shape),
            ds.reshape(scales.shape), None, None, None)


torch.library.register_autograd("flash_prologue::qknorm_rope_scale", _backward,
                                setup_context=_setup_context)
