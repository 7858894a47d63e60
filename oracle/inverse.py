"""Restatement of the reference's inverse (recompute-from-outputs) prologue -- TEST ORACLE.

TEST INFRASTRUCTURE: only tests/ may use it, as the checker.

Reference: flash_attn_prologue/fused_epilogue.py
* forward ``qknorm_rope_scale_cute_inverse`` (:2560-2653, kernel :1663-1992):
  the outputs of the ``native`` formulation plus, per row, the statistic
  r = rsqrt(sum(x^2)/D + eps) (:1913-1917), FP32 ``[B, H, N, 1]``;
* backward ``qknorm_rope_scale_cute_inverse_backward`` (:2671-2772, kernel
  :2067-2358, arithmetic :2196-2300), restated op for op in FP32:
    u   = out / e                    (Q only; e = exp(scale[h]))
    m   = R^T u                      (m1 = u1 c + u2 s, m2 = u2 c - u1 s)
    n   = m / w                      ("normed" = x * r)
    g'  = grad_out * e               (Q only)
    dy  = R^T g'
    rot = R(n * w)
    ds[h]  += sum_j g'_j rot_j       (Q rows)
    dw[t]  += dy * n                 (summed over all rows)
    dx  = r * (dy * w - n * sum_j(dy_j w_j n_j) / D)

All tensors are 4-D ``[B, H, N, D]`` (the raw op's view); sin/cos broadcast as
``[B|1, 1, N|1, D/2]``. Pinning: the forward is the ``native`` restatement
(pinned to the reference-generated golden vectors) plus r; the backward is
pinned through the golden vectors by the identity it relies on -- fed the
outputs of the FP32 golden cases it must reproduce the reference's autograd
gradients (tests/test_oracle_inverse.py).
"""
import torch

from .native import native_forward


def inverse_forward(q, k, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    """(q_out, k_out, rms_q, rms_k) of the inverse forward on 4-D inputs."""
    q_out, k_out = native_forward(q, k, rmsnorm_weight, scales, sin, cos, eps=eps)
    d = q.shape[-1]

    def stat(x):
        x = x.float()
        return torch.rsqrt(x.square().sum(-1, keepdim=True) / d + eps)

    return q_out, k_out, stat(q), stat(k)


def _rope(a1, a2, c, s):
    return a1 * c - a2 * s, a2 * c + a1 * s


def _rope_t(a1, a2, c, s):
    return a1 * c + a2 * s, a2 * c - a1 * s


def inverse_backward(q_out, k_out, rmsnorm_weight, scales, sin, cos, grad_q_out, grad_k_out,
                     rms_q, rms_k):
    """(dq, dk, dw [2,1,D], ds [H,1,1]) of the inverse backward, FP32 arithmetic."""
    d = q_out.shape[-1]
    half = d // 2
    c, s = cos.float(), sin.float()
    e = torch.exp(scales.float().reshape(1, -1, 1, 1))
    grads, dws, ds = [], [], None
    for t, (out, g, r) in enumerate(((q_out, grad_q_out, rms_q), (k_out, grad_k_out, rms_k))):
        w = rmsnorm_weight[t].float().reshape(-1)
        u = out.float() / e if t == 0 else out.float()
        m1, m2 = _rope_t(u[..., :half], u[..., half:], c, s)
        n = torch.cat((m1 / w[:half], m2 / w[half:]), dim=-1)
        gp = g.float() * e if t == 0 else g.float()
        dy = torch.cat(_rope_t(gp[..., :half], gp[..., half:], c, s), dim=-1)
        a = n * w
        rot = torch.cat(_rope(a[..., :half], a[..., half:], c, s), dim=-1)
        if t == 0:
            ds = (gp * rot).sum(-1).sum((0, 2)).reshape(-1, 1, 1)
        dws.append((dy * n).reshape(-1, d).sum(0))
        total = (dy * w * n).sum(-1, keepdim=True)
        dx = r.float() * (dy * w - n * (total / d))
        grads.append(dx.to(out.dtype))
    return grads[0], grads[1], torch.stack(dws).reshape(2, 1, d), ds
