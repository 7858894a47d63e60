"""``FusedQKV`` module (reference: flash_attn_prologue/layers/FusedQKV.py:170-205).

CPU: constructor, parameter names/shapes/initial values, the missing-thetas and
dtype errors. GPU: forward and backward of the module against the eager FP32
formulation F.linear -> RMSNorm -> split-half RoPE -> Q * exp(scale) (each
projection rounded to BF16 first, as the kernel's BF16 GEMM output is), at
the module test's tolerances (rtol 1e-2, atol 1e-1 on BF16 outputs; relative
error on gradients), with half- and full-width (rotate-half) RoPE tables and
a non-default eps.
"""
import math

import pytest
import torch

from flash_attn_prologue_b200 import FusedQKV
from tests._util import rel_err


def test_parameters_and_initial_values():
    m = FusedQKV(hidden_size=256, num_heads=4, head_dim=64)
    names = dict(m.named_parameters())
    assert set(names) == {"qkv_proj.weight", "qk_norm_weight", "scales"}
    assert names["qkv_proj.weight"].shape == (3 * 4 * 64, 256)
    assert m.qkv_proj.bias is None
    assert torch.equal(m.qk_norm_weight, torch.ones(2, 1, 64))
    assert torch.allclose(m.scales, torch.full((4, 1, 1), math.log(64 ** -0.5)))
    assert float(m.qkv_proj.weight.detach().std()) < 0.03


def test_errors():
    m = FusedQKV(256, 4, 64)
    x = torch.randn(1, 8, 256)
    with pytest.raises(ValueError, match="thetas"):
        m(x)
    with pytest.raises(ValueError, match="BF16"):
        m(x, (torch.zeros(8, 32), torch.ones(8, 32)))
    with pytest.raises(ValueError):
        FusedQKV(256, 4, 63)


def _eager(x, weight, w, s, sin, cos, H, D, eps):
    B, N, _ = x.shape
    p = torch.nn.functional.linear(x, weight).view(B, N, 3, H, D).permute(2, 0, 3, 1, 4)
    outs = []
    for i in range(2):
        t = p[i].float()
        n = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w[i, 0]
        a, b = n.chunk(2, dim=-1)
        r = torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)
        if i == 0:
            r = r * s.float().exp()
        outs.append(r.to(x.dtype))
    return outs[0], outs[1], p[2]


@pytest.mark.gpu
@pytest.mark.parametrize("full_width", [False, True])
@pytest.mark.parametrize("D,eps", [(64, 1e-5), (128, 1e-3)])
def test_forward_backward_against_eager(D, eps, full_width):
    torch.manual_seed(D)
    B, N, hidden, H = 2, 96, 256, 4
    m = FusedQKV(hidden, H, D, eps=eps).to(device="cuda", dtype=torch.bfloat16)
    x = torch.randn(B, N, hidden, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    ang = torch.randn(N, D // 2, device="cuda")
    sin, cos = ang.sin(), ang.cos()
    thetas = (torch.cat((sin, sin), -1), torch.cat((cos, cos), -1)) if full_width else (sin, cos)
    q, k, v = m(x, thetas)
    assert q.shape == k.shape == v.shape == (B, H, N, D) and q.is_contiguous()
    xr = x.detach().clone().requires_grad_()
    wr = m.qkv_proj.weight.detach().clone().requires_grad_()
    nw = m.qk_norm_weight.detach().float().clone().requires_grad_()
    sc = m.scales.detach().float().clone().requires_grad_()
    qe, ke, ve = _eager(xr, wr, nw, sc, sin, cos, H, D, eps)
    for got, exp in ((q, qe), (k, ke), (v, ve)):
        torch.testing.assert_close(got, exp, rtol=1e-2, atol=1e-1)
    g = [torch.randn_like(t) for t in (q, k, v)]
    grads = torch.autograd.grad((q, k, v), (x, m.qkv_proj.weight, m.qk_norm_weight, m.scales), g)
    grads_e = torch.autograd.grad((qe, ke, ve), (xr, wr, nw, sc), g)
    for a, b in zip(grads, grads_e):
        assert rel_err(a.float(), b.float()) < 2e-2
