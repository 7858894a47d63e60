"""The reference's projection-backward tests at their own shapes and tolerances.

* tests/test_gemm_bwd_clone.py: B = 32, N = 512, hidden = 512, H = 16, D = 64,
  truncated-normal (std 0.3) gradients, weight and x; matmul_bwd_dx_cute and
  matmul_bwd_dw_cute against the BF16 eager products (here: against the FP32
  products, 1 BF16 ulp or the FP32 rounding band of the terms);
* tests/test_fused_qkv_extras.py: empty inputs (N = 0) through fused_qkv,
  fused_qkv_backward, matmul_bwd_dx_cute, matmul_bwd_dw and a
  torch.compile(fullgraph=True) function of them; and in-place accumulation of
  matmul_bwd_dw into zero / random ``out`` (rtol 2e-2, atol 1e-1), eager and
  compiled.
"""
import math

import pytest
import torch

import flash_attn_prologue_b200 as fap
from flash_attn_prologue_b200 import gemm_bwd

pytestmark = pytest.mark.gpu
OPS = torch.ops.flash_prologue


def _truncated_normal(shape, std, g):
    # inverse-CDF sampling restricted to [-2 std, 2 std]
    u = torch.rand(shape, generator=g, device="cuda")
    lo, hi = 0.5 * (1 + math.erf(-2 / math.sqrt(2))), 0.5 * (1 + math.erf(2 / math.sqrt(2)))
    u = lo + u * (hi - lo)
    return (math.sqrt(2.0) * torch.erfinv(2.0 * u - 1.0) * std).to(torch.bfloat16)


def _within_band(got, a, b):
    """1 BF16 ulp of the FP32 product rounded to BF16, or the FP32 rounding band of its terms."""
    from tests.test_qkv_backward_ops import _check_gemm
    _check_gemm(got, a.float(), b.float())


def test_cloned_gemm_bwd_shapes():
    B, N, hidden, H, D = 32, 512, 512, 16, 64
    g = torch.Generator(device="cuda").manual_seed(42)
    grad_output = _truncated_normal((B * N, 3 * H * D), 0.3, g)
    weight = _truncated_normal((3 * H * D, hidden), 0.3, g)
    x = _truncated_normal((B * N, hidden), 0.3, g)
    qkv = grad_output.view(B, N, 3, H, D)
    gq, gk, gv = (qkv[..., i, :, :].permute(0, 2, 1, 3).contiguous() for i in range(3))
    dx = OPS.matmul_bwd_dx_cute(gq, gk, gv, weight)
    dw = OPS.matmul_bwd_dw_cute(gq, gk, gv, x)
    assert dx.shape == (B * N, hidden) and dw.shape == (3 * H * D, hidden)
    assert not torch.isnan(dx).any() and not torch.isnan(dw).any()
    _within_band(dx, grad_output, weight)
    _within_band(dw, grad_output.t(), x)


def test_empty_inputs_including_compiled():
    B, N, hidden, H, D = 32, 0, 512, 16, 64
    x = torch.zeros((B, N, hidden), device="cuda", dtype=torch.bfloat16)
    w = torch.zeros((3 * H * D, hidden), device="cuda", dtype=torch.bfloat16)
    q, k, v = OPS.fused_qkv(x, w)
    assert q.shape == k.shape == v.shape == (B, H, N, D) and q.numel() == 0
    zeros = [torch.zeros((B, H, N, D), device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    dx, dw = OPS.fused_qkv_backward(*zeros, w, x)
    assert dx.shape == (B, N, hidden) and dw.shape == (3 * H * D, hidden)
    assert float(dw.abs().sum()) == 0.0
    assert OPS.matmul_bwd_dx_cute(*zeros, w).shape == (0, hidden)
    assert float(gemm_bwd.matmul_bwd_dw(*zeros, x).abs().sum()) == 0.0

    @torch.compile(fullgraph=True)
    def compiled(xv, wv):
        qv, kv, vv = OPS.fused_qkv(xv, wv)
        return qv, *OPS.fused_qkv_backward(torch.zeros_like(qv), torch.zeros_like(kv),
                                           torch.zeros_like(vv), wv, xv)

    qc, dxc, dwc = compiled(x, w)
    assert qc.numel() == 0 and dxc.numel() == 0 and float(dwc.abs().sum()) == 0.0


def test_inplace_accumulation_eager_and_compiled():
    B, N, hidden, H, D = 4, 128, 128, 4, 64
    g = torch.Generator(device="cuda").manual_seed(42)
    gq, gk, gv = (torch.randn((B, H, N, D), generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    x = torch.randn((B, N, hidden), generator=g, device="cuda").to(torch.bfloat16)
    ref = gemm_bwd.matmul_bwd_dw(gq, gk, gv, x)
    out0 = torch.zeros_like(ref)
    res0 = gemm_bwd.matmul_bwd_dw(gq, gk, gv, x, out=out0)
    assert res0 is out0
    torch.testing.assert_close(out0, ref, atol=1e-1, rtol=2e-2)
    out1 = torch.randn(ref.shape, generator=g, device="cuda").to(torch.bfloat16)
    expect = out1.clone() + ref
    gemm_bwd.matmul_bwd_dw(gq, gk, gv, x, out=out1)
    torch.testing.assert_close(out1, expect, atol=1e-1, rtol=2e-2)

    @torch.compile(fullgraph=True)
    def compiled(a, b, c, xv, o):
        return gemm_bwd.matmul_bwd_dw(a, b, c, xv, out=o)

    out2 = torch.randn(ref.shape, generator=g, device="cuda").to(torch.bfloat16)
    expect2 = out2.clone() + ref
    res2 = compiled(gq, gk, gv, x, out2)
    torch.testing.assert_close(res2, expect2, atol=1e-1, rtol=2e-2)
    torch.testing.assert_close(out2, expect2, atol=1e-1, rtol=2e-2)
