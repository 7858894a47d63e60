"""Independent float64 oracle (numpy) for the prologue forward and backward.

Forward follows the reference tests' FP64 oracle (tests/test_frontend_api.py:13-32):
RMS from the vector norm, weights applied, then an explicit 2x2 rotation of
each (j, j+D/2) pair, Q times exp(scale). Backward is the closed form used by
the reference backward kernel (flash_attn_prologue/fused_epilogue.py:1047-1126):

    r = (mean(x^2) + eps)^-1/2,  n = x r,  g' = g * exp(s) (Q) or g (K)
    dn = R^T g'                           (inverse rotation)
    dw[t] = sum over rows of dn * n
    ds[h] = sum over Q rows of head h of g' . R (n w)
    dx = r (dn w - n mean(dn w n))

Arrays are dense [B, H, N, D] float64 (packed [T,H,D] callers pass B=1 after
transposing); sin/cos broadcast to [B, 1, N, D/2]. TEST INFRASTRUCTURE.
"""
import numpy as np


def _rows(x):
    return np.asarray(x, dtype=np.float64)


def fp64_forward(q, k, w, s, sin, cos, eps=1e-5):
    """q, k: [B,H,N,D]; w: [2,1,D]; s: [H]; sin/cos: broadcastable to [B,1,N,D/2]."""
    q, k, w, s = _rows(q), _rows(k), _rows(w), _rows(s).reshape(-1)
    sin, cos = _rows(sin), _rows(cos)
    outs = []
    for t, x in enumerate((q, k)):
        d = x.shape[-1]
        rms = np.sqrt(np.linalg.norm(x, axis=-1, keepdims=True) ** 2 / d + eps)
        y = x / rms * w[t].reshape(1, 1, 1, d)
        a, b = y[..., : d // 2], y[..., d // 2:]
        out = np.concatenate((a * cos - b * sin, a * sin + b * cos), axis=-1)
        if t == 0:
            out = out * np.exp(s).reshape(1, -1, 1, 1)
        outs.append(out)
    return tuple(outs)


def fp64_backward(q, k, w, s, sin, cos, gq, gk, eps=1e-5):
    """Returns (dq, dk, dw [2,1,D], ds [H,1,1]) in float64."""
    q, k, w, s = _rows(q), _rows(k), _rows(w), _rows(s).reshape(-1)
    sin, cos = _rows(sin), _rows(cos)
    gq, gk = _rows(gq), _rows(gk)
    d = q.shape[-1]
    h2 = d // 2
    dx_all, dw = [], np.zeros((2, 1, d))
    ds = np.zeros((q.shape[1], 1, 1))
    for t, (x, g) in enumerate(((q, gq), (k, gk))):
        r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
        n = x * r
        wt = w[t].reshape(1, 1, 1, d)
        if t == 0:
            g = g * np.exp(s).reshape(1, -1, 1, 1)
        g1, g2 = g[..., :h2], g[..., h2:]
        dn = np.concatenate((g1 * cos + g2 * sin, g2 * cos - g1 * sin), axis=-1)
        dw[t, 0] = (dn * n).reshape(-1, d).sum(0)
        if t == 0:
            y = n * wt
            a, b = y[..., :h2], y[..., h2:]
            rot = np.concatenate((a * cos - b * sin, a * sin + b * cos), axis=-1)
            ds[:, 0, 0] = (g * rot).sum(axis=(0, 2, 3))
        dnw = dn * wt
        dx_all.append(r * (dnw - n * (dnw * n).mean(-1, keepdims=True)))
    return dx_all[0], dx_all[1], dw, ds
