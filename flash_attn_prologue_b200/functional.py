"""Q/K RMSNorm -> split-half RoPE -> query scale: the public functional API.

Same signature, validation order, messages and layouts as the reference
frontend (flash_attn_prologue/functional.py:6-94). ``backend="cute"`` runs the
sm_100a CUDA kernels of libflash_prologue.so through the
``flash_prologue::qknorm_rope_scale_cute`` custom op; ``backend="native"`` is
the reference's own traceable PyTorch formulation, kept so callers that select
it by name keep working. The two are separate choices made by the caller:
the ``cute`` path never routes to ``native`` (empty inputs included).
"""
import math

import torch

SUPPORTED_CUTE_HEAD_DIMS = (32, 64, 128, 256)
_CUTE_DTYPES = (torch.bfloat16, torch.float16, torch.float32)


def prepare_backend(backend: str = "native") -> None:
    """Registers the CUDA custom ops before a compiled graph is captured."""
    if backend not in ("native", "cute"):
        raise ValueError("backend must be 'native' or 'cute'")
    if backend == "cute":
        from . import fused_epilogue  # noqa: F401


def qknorm_rope_scale(q, k, rmsnorm_weight, scales, sin, cos, eps=1e-5, *, backend="native"):
    """Normalize Q/K, apply half-width RoPE, and multiply Q by exp(scales).

    Q/K: matching packed [T,H,D] or dense [B,H,N,D], BF16/FP16/FP32.
    Weight: [2,1,D]. Log-scales: [H,1,1]. Both must be FP32.
    Packed sin/cos: [T,D/2] or [T,1,D/2]. Dense: [N,D/2], [B,N,D/2], or
    [B,1,N,D/2]; singleton B/N broadcasting is supported. Frequencies are FP32;
    positions and RoPE resets are the caller's (per-row op: no cu_seqlens).
    All arithmetic through the final cast is FP32. Inputs are never mutated.
    ``cute``: CUDA, BF16/FP16/FP32, D in (32, 64, 128, 256), up to 512 heads,
    any eps > 0; no sin/cos gradients. Strided q/k views (e.g. slices of a
    fused QKV buffer) are read in place.
    """
    if backend not in ("native", "cute"):
        raise ValueError("backend must be 'native' or 'cute'")
    if q.ndim not in (3, 4) or q.shape != k.shape:
        raise ValueError("q/k must have matching packed [T,H,D] or dense [B,H,N,D] shapes")
    if q.dtype not in (torch.bfloat16, torch.float16, torch.float32) or k.dtype != q.dtype:
        raise ValueError("q/k must share BF16, FP16, or FP32 dtype")
    d, h = q.shape[-1], q.shape[-2] if q.ndim == 3 else q.shape[1]
    if d <= 0 or d % 2 or h <= 0:
        raise ValueError("head dimension must be positive/even and head count positive")
    if not math.isfinite(eps) or eps <= 0:
        raise ValueError("eps must be finite and positive")
    if rmsnorm_weight.shape != (2, 1, d) or scales.shape != (h, 1, 1):
        raise ValueError("weight must be [2,1,D], log-scales must be [H,1,1]")
    for value in (rmsnorm_weight, scales, sin, cos):
        if value.dtype != torch.float32:
            raise ValueError("weights, log-scales, and sin/cos must be FP32")
    if any(t.device != q.device for t in (k, rmsnorm_weight, scales, sin, cos)):
        raise ValueError("all tensors must share a device")
    if sin.shape != cos.shape or sin.shape[-1:] != (d // 2,):
        raise ValueError("sin/cos must have identical shapes and half-width D/2")
    if q.ndim == 3:
        if sin.ndim == 2:
            sin, cos = sin[:, None, :], cos[:, None, :]
        if sin.ndim != 3 or sin.shape[0] not in (1, q.shape[0]) or sin.shape[1] != 1:
            raise ValueError("packed sin/cos must be [T,D/2] or [T,1,D/2]")
        scale = scales.reshape(1, h, 1)
    else:
        if sin.ndim == 2:
            sin, cos = sin[None, None, :, :], cos[None, None, :, :]
        elif sin.ndim == 3:
            sin, cos = sin[:, None, :, :], cos[:, None, :, :]
        if (sin.ndim != 4 or sin.shape[0] not in (1, q.shape[0])
                or sin.shape[1] != 1 or sin.shape[2] not in (1, q.shape[2])):
            raise ValueError("dense sin/cos must broadcast over [B,1,N,D/2]")
        scale = scales[None, :, :, :]
    if backend == "cute":
        if q.device.type != "cuda" or q.dtype not in _CUTE_DTYPES or d not in SUPPORTED_CUTE_HEAD_DIMS:
            raise ValueError("CuTe requires CUDA q/k and D in (32, 64, 128, 256)")
        if h > 512:
            raise ValueError("CuTe supports at most 512 heads")
        if sin.requires_grad or cos.requires_grad:
            raise ValueError("CuTe does not implement frequency gradients; use native")
        prepare_backend("cute")
        if q.ndim == 3:
            q4, k4 = q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None]
            s4, c4 = sin.permute(1, 0, 2)[None], cos.permute(1, 0, 2)[None]
        else:
            q4, k4, s4, c4 = q, k, sin, cos
        s4 = s4.expand(q4.shape[0], 1, q4.shape[2], d // 2)
        c4 = c4.expand_as(s4)
        if q4.stride(-1) != 1 or any(n > 1 and st == 0 for n, st in zip(q4.shape, q4.stride())):
            q4 = q4.contiguous()
        if k4.stride(-1) != 1 or any(n > 1 and st == 0 for n, st in zip(k4.shape, k4.stride())):
            k4 = k4.contiguous()
        out_q, out_k = torch.ops.flash_prologue.qknorm_rope_scale_cute(
            q4, k4, rmsnorm_weight, scales, s4, c4, eps)
        if q.ndim == 3:
            # squeeze (a view in both directions), not out[0]: the backward of a
            # select would allocate zeros and scatter-copy every gradient.
            return out_q.squeeze(0).permute(1, 0, 2), out_k.squeeze(0).permute(1, 0, 2)
        return out_q, out_k

    def transform(x, weight):
        x = x.float()
        normed = x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * weight
        first, second = normed.chunk(2, dim=-1)
        return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)

    return ((transform(q, rmsnorm_weight[0]) * scale.exp()).to(q.dtype),
            transform(k, rmsnorm_weight[1]).to(k.dtype))
