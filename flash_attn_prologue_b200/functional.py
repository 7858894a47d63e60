"""Q/K RMSNorm -> split-half RoPE -> query scale: the public functional API.

Same signature, validation order, messages and layouts as the reference
frontend (flash_attn_prologue/functional.py:6-94). ``backend="cute"`` runs the
sm_100a CUDA kernels of libflash_prologue.so through the
``flash_prologue::qknorm_rope_scale_cute`` custom op (plain eager calls take
the op's own body directly, skipping the dispatch layers); ``backend="native"`` is
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


def _validate(q, k, rmsnorm_weight, scales, sin, cos, eps, backend):
    """The reference frontend's checks, in its order (functional.py:29-70).

    Returns sin/cos reshaped for broadcasting against q/k and the scale view
    of the native formulation; raises the reference's ValueError texts.
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
    return sin, cos, scale


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
    sin, cos, scale = _validate(q, k, rmsnorm_weight, scales, sin, cos, eps, backend)
    if backend == "cute":
        prepare_backend("cute")
        d = q.shape[-1]
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
        if _plain_eager(q4, k4, rmsnorm_weight, scales, s4, c4):
            out_q, out_k = _CuteEager.apply(q4, k4, rmsnorm_weight, scales, s4, c4, eps)
        else:
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


def _plain_eager(*tensors) -> bool:
    """True for an eager call on plain tensors: not compiled, traced, under a
    functorch transform or on tensor subclasses (fake, meta wrappers, DTensor),
    where the registered custom op must be what is recorded."""
    if torch.compiler.is_compiling() or torch.jit.is_tracing():
        return False
    active = getattr(torch._C, "_are_functorch_transforms_active", None)
    if active is not None and active():
        return False
    return all(type(t) is torch.Tensor for t in tensors)


class _CuteEager(torch.autograd.Function):
    """qknorm_rope_scale_cute for eager calls without the custom-op dispatch
    layers (tens of microseconds on small problems): the same forward and
    backward bodies (fused_epilogue.cute_forward / cute_backward), so the
    same kernels and results as the registered op and its autograd."""

    @staticmethod
    def forward(ctx, q, k, rmsnorm_weight, scales, sin, cos, eps):
        from .fused_epilogue import cute_forward
        ctx.save_for_backward(q, k, rmsnorm_weight, scales, sin, cos)
        ctx.eps = eps
        return cute_forward(q, k, rmsnorm_weight, scales, sin, cos, eps)

    @staticmethod
    def backward(ctx, grad_q, grad_k):
        from .fused_epilogue import cute_backward
        q, k, rmsnorm_weight, scales, sin, cos = ctx.saved_tensors
        dq, dk, dw, ds = cute_backward(q, k, rmsnorm_weight, scales, sin, cos, grad_q, grad_k, ctx.eps)
        return dq, dk, dw, ds, None, None, None


def _cute_tables(sin, cos, packed, B, N, half):
    """sin/cos (as reshaped by _validate) as [B|1, 1, N, D/2] views for the op."""
    if packed:
        sin, cos = sin.permute(1, 0, 2)[None], cos.permute(1, 0, 2)[None]
    sin = sin.expand(sin.shape[0], 1, N, half)
    return sin, cos.expand_as(sin)


class _QKVPrologue(torch.autograd.Function):
    """Prologue on the Q/K slots of a packed QKV tensor, V passed through.

    The backward writes dq, dk and dv straight into one gradient tensor laid
    out like qkv, instead of autograd gathering three separate gradients of
    slice views into it (which re-reads and re-writes dq and dk).
    """

    @staticmethod
    def forward(ctx, qkv5, rmsnorm_weight, scales, sin4, cos4, eps):
        q4 = qkv5[:, :, 0].permute(0, 2, 1, 3)
        k4 = qkv5[:, :, 1].permute(0, 2, 1, 3)
        out_q, out_k = torch.ops.flash_prologue.qknorm_rope_scale_cute(
            q4, k4, rmsnorm_weight, scales, sin4, cos4, eps)
        ctx.save_for_backward(qkv5, rmsnorm_weight, scales, sin4, cos4)
        ctx.eps = eps
        return out_q, out_k, qkv5[:, :, 2].permute(0, 2, 1, 3)

    @staticmethod
    def backward(ctx, grad_q, grad_k, grad_v):
        qkv5, rmsnorm_weight, scales, sin4, cos4 = ctx.saved_tensors
        gv = None if grad_v is None else grad_v.permute(0, 2, 1, 3)
        grad_qkv, dw, ds = torch.ops.flash_prologue.qknorm_rope_scale_qkv_backward(
            qkv5, rmsnorm_weight, scales, sin4, cos4, grad_q, grad_k, gv, ctx.eps)
        return grad_qkv, dw, ds, None, None, None


def qknorm_rope_scale_qkv(qkv, rmsnorm_weight, scales, sin, cos, eps=1e-5, *, backend="cute"):
    """qknorm_rope_scale on the Q and K slots of a fused QKV activation; returns (q, k, v).

    qkv: packed [T, 3, H, D] or batched [B, N, 3, H, D] (a QKV projection's
    output viewed as heads; slot 0 = Q, 1 = K, 2 = V). Returns q_out, k_out and
    v in the layouts of qknorm_rope_scale: packed [T, H, D], batched
    [B, H, N, D] (v is a view of qkv). Other arguments and checks as
    qknorm_rope_scale. With ``cute`` the backward produces the gradient of qkv
    as one tensor: the kernel writes dq and dk into its Q and K slots and the
    gradient of v lands in its V slot (zeros when v is unused), so no
    per-slice gradients are gathered afterwards. ``native`` is the reference
    formulation on the unbound slices.
    """
    if qkv.ndim not in (4, 5) or qkv.shape[-3] != 3:
        raise ValueError("qkv must be packed [T,3,H,D] or batched [B,N,3,H,D]")
    packed = qkv.ndim == 4
    q, k, v = qkv.unbind(-3)
    if not packed:
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    sin, cos, _ = _validate(q, k, rmsnorm_weight, scales, sin, cos, eps, backend)
    if backend == "native":
        q_out, k_out = qknorm_rope_scale(q, k, rmsnorm_weight, scales, sin, cos, eps, backend="native")
        return q_out, k_out, v
    prepare_backend("cute")
    qkv5 = qkv[None] if packed else qkv
    if qkv5.stride(-1) != 1:
        qkv5 = qkv5.contiguous()
    B, N, _, H, D = qkv5.shape
    sin4, cos4 = _cute_tables(sin, cos, packed, B, N, D // 2)
    out_q, out_k, v4 = _QKVPrologue.apply(qkv5, rmsnorm_weight, scales, sin4, cos4, eps)
    if packed:
        return (out_q.squeeze(0).permute(1, 0, 2), out_k.squeeze(0).permute(1, 0, 2),
                v4.squeeze(0).permute(1, 0, 2))
    return out_q, out_k, v4
