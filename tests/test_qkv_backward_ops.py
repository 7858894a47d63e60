"""Backward ops of the fused QKV projection under the reference's names.

``fused_qkv_backward``, ``matmul_bwd_dx_cute``, ``matmul_bwd_dw_cute`` /
``matmul_bwd_dw_accumulate_cute`` and the Python ``matmul_bwd_dw`` (reference:
flash_attn_prologue/gemm_bwd.py:1171-1566; tests/test_fused_qkv_extras.py for
empty inputs and in-place accumulation) are checked on CPU against the FP32
formulation dX = dP W, dW = dP^T X with dP the per-head gradients laid out as
the [B*N, 3*H*D] projection gradient. GPU: ``fused_qkv_epilogue_ckp`` (the
recompute composite, reference fused_qkv.py:880-1053) gives outputs and
gradients bit-identical to ``fused_qkv_epilogue``.
"""
import math

import pytest
import torch

import flash_attn_prologue_b200 as fap
from tests._util import rel_err

OPS = torch.ops.flash_prologue


def _grads(B, H, N, D, hidden, seed=0, device="cpu", dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    gq, gk, gv = (torch.randn(B, H, N, D, generator=g).to(dtype).to(device) for _ in range(3))
    x = torch.randn(B, N, hidden, generator=g).to(dtype).to(device)
    w = (0.02 * torch.randn(3 * H * D, hidden, generator=g)).to(dtype).to(device)
    return gq, gk, gv, x, w


def _dp(gq, gk, gv):
    B, H, N, D = gq.shape
    return torch.stack((gq, gk, gv), 0).permute(1, 3, 0, 2, 4).reshape(B * N, 3 * H * D).float()


@pytest.mark.parametrize("B,H,N,D,hidden", [(2, 4, 16, 64, 128), (1, 2, 33, 128, 64)])
def test_fused_qkv_backward_matches_fp32_formulation(B, H, N, D, hidden):
    gq, gk, gv, x, w = _grads(B, H, N, D, hidden, seed=N)
    grad_x, grad_w = fap.fused_qkv_backward(gq, gk, gv, w, x)
    dp = _dp(gq, gk, gv)
    assert grad_x.shape == (B, N, hidden) and grad_w.shape == (3 * H * D, hidden)
    assert rel_err(grad_x.float(), (dp @ w.float()).reshape(B, N, hidden)) < 1e-2
    assert rel_err(grad_w.float(), dp.t() @ x.float().reshape(B * N, hidden)) < 1e-2
    dx = OPS.matmul_bwd_dx_cute(gq, gk, gv, w)
    assert dx.shape == (B * N, hidden) and torch.equal(dx.reshape(B, N, hidden), grad_x)
    assert torch.equal(fap.matmul_bwd_dw(gq, gk, gv, x), grad_w)


def test_matmul_bwd_dw_accumulates_in_place():
    gq, gk, gv, x, w = _grads(2, 2, 8, 64, 64, seed=5, dtype=torch.float32)
    out = torch.randn(3 * 2 * 64, 64)
    before = out.clone()
    ret = fap.matmul_bwd_dw(gq, gk, gv, x, out=out)
    assert ret is out
    expect = before + _dp(gq, gk, gv).t() @ x.reshape(-1, 64)
    torch.testing.assert_close(out, expect, rtol=1e-5, atol=1e-5)


def test_empty_inputs_give_zero_gradients():
    gq, gk, gv, x, w = _grads(3, 4, 0, 64, 128)
    grad_x, grad_w = fap.fused_qkv_backward(gq, gk, gv, w, x)
    assert grad_x.shape == (3, 0, 128) and grad_w.shape == (3 * 4 * 64, 128)
    assert float(grad_w.abs().sum()) == 0.0
    assert OPS.matmul_bwd_dx_cute(gq, gk, gv, w).shape == (0, 128)
    assert float(fap.matmul_bwd_dw(gq, gk, gv, x).abs().sum()) == 0.0


def test_opcheck_schemas():
    gq, gk, gv, x, w = _grads(1, 2, 4, 64, 64, dtype=torch.float32)
    torch.library.opcheck(OPS.fused_qkv_backward, (gq, gk, gv, w, x))
    torch.library.opcheck(OPS.matmul_bwd_dx_cute, (gq, gk, gv, w))
    torch.library.opcheck(OPS.matmul_bwd_dw_cute, (gq, gk, gv, x))


def _problem(B, N, hidden, H, D, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, N, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(3 * H * D, hidden, generator=g, device="cuda")).to(torch.bfloat16)
    rw = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    sc = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda") - math.log(D) / 2
    ang = torch.rand(N, D // 2, generator=g, device="cuda") * 6.0
    return x, w, rw, sc, ang.sin(), ang.cos()


@pytest.mark.gpu
@pytest.mark.parametrize("B,N,hidden,H,D", [(2, 128, 256, 2, 128), (1, 200, 128, 4, 64)])
def test_checkpoint_composite_equals_saving_composite(B, N, hidden, H, D):
    x, w, rw, sc, sin, cos = _problem(B, N, hidden, H, D, seed=N)
    g = torch.Generator(device="cuda").manual_seed(1)
    gq, gk, gv = (torch.randn(B, H, N, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    results = []
    for op in (fap.fused_qkv_epilogue, fap.fused_qkv_epilogue_ckp):
        leaves = [t.detach().clone().requires_grad_(i < 4) for i, t in enumerate((x, w, rw, sc, sin, cos))]
        outs = op(*leaves)[:3]
        grads = torch.autograd.grad(outs, leaves[:4], (gq, gk, gv))
        results.append((outs, grads))
    torch.cuda.synchronize()
    for a, b in zip(results[0][0] + results[0][1], results[1][0] + results[1][1]):
        assert torch.equal(a, b)
