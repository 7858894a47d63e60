"""Restatement of the reference ``native`` backend on CPU tensors (test oracle).

Reference: flash_attn_prologue/functional.py:49-63 (packed/dense sin/cos
broadcasting, scale reshape) and :89-94 (the arithmetic):

    x = x.float()
    normed = x * rsqrt(mean(x^2, -1) + eps) * weight
    first, second = chunk(normed, 2)
    out = cat(first*cos - second*sin, second*cos + first*sin)
    q_out = (out_q * exp(scale)).to(dtype);  k_out = out_k.to(dtype)

The backward is autograd through exactly these ops, as in the reference.
TEST INFRASTRUCTURE: not used by the product path.
"""
import torch


def _broadcast_tables(q, sin, cos, scales):
    """functional.py:49-63: table and scale shapes for packed [T,H,D] / dense [B,H,N,D]."""
    h = q.shape[-2] if q.ndim == 3 else q.shape[1]
    if q.ndim == 3:
        if sin.ndim == 2:
            sin, cos = sin[:, None, :], cos[:, None, :]
        scale = scales.reshape(1, h, 1)
    else:
        if sin.ndim == 2:
            sin, cos = sin[None, None, :, :], cos[None, None, :, :]
        elif sin.ndim == 3:
            sin, cos = sin[:, None, :, :], cos[:, None, :, :]
        scale = scales[None, :, :, :]
    return sin, cos, scale


def native_forward(q, k, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    """Forward of the reference ``native`` backend (CPU or any device tensors)."""
    sin, cos, scale = _broadcast_tables(q, sin, cos, scales)

    def transform(x, weight):
        x = x.float()
        normed = x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * weight
        first, second = normed.chunk(2, dim=-1)
        return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)

    return ((transform(q, rmsnorm_weight[0]) * scale.exp()).to(q.dtype),
            transform(k, rmsnorm_weight[1]).to(k.dtype))


def native_forward_backward(q, k, rmsnorm_weight, scales, sin, cos, grad_q_out, grad_k_out,
                            eps=1e-5):
    """Outputs and (dq, dk, dw, ds) of the native path for given upstream gradients."""
    args = [t.detach().clone().requires_grad_(i < 4) for i, t in
            enumerate((q, k, rmsnorm_weight, scales, sin, cos))]
    outs = native_forward(*args, eps=eps)
    grads = torch.autograd.grad(outs, args[:4], (grad_q_out, grad_k_out))
    return tuple(o.detach() for o in outs), tuple(grads)
