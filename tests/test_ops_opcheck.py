"""torch.library.opcheck and torch.compile(fullgraph=True) over every custom op of the package.

opcheck runs each op's schema, fake-tensor and autograd-registration checks
(as the reference's cute op is checked in tests/test_frontend_api.py); the
compiled runs trace the forward and backward of the composite entry points
into one graph and must reproduce the eager results bit for bit.
"""
import math

import pytest
import torch

import flash_attn_prologue_b200 as fap
from flash_attn_prologue_b200 import fused_epilogue, fused_qkv  # noqa: F401  (register the ops)

pytestmark = pytest.mark.gpu
OPS = torch.ops.flash_prologue
CHECKS = ("test_schema", "test_autograd_registration", "test_faketensor")


def _prologue_args(B=2, H=4, N=24, D=64, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g, device="cuda").to(torch.bfloat16).requires_grad_()
    k = torch.randn(B, H, N, D, generator=g, device="cuda").to(torch.bfloat16).requires_grad_()
    w = (1 + 0.1 * torch.randn(2, 1, D, generator=g, device="cuda")).requires_grad_()
    s = (0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")).requires_grad_()
    ang = torch.rand(1, 1, N, D // 2, generator=g, device="cuda") * 3
    return q, k, w, s, ang.sin(), ang.cos()


def _gemm_args(B=1, N=128, hidden=128, H=2, D=128, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, N, hidden, generator=g, device="cuda").to(torch.bfloat16).requires_grad_()
    w = (0.02 * torch.randn(3 * H * D, hidden, generator=g, device="cuda")).to(torch.bfloat16).requires_grad_()
    rw = (1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")).requires_grad_()
    sc = (0.1 * torch.randn(H, 1, 1, generator=g, device="cuda") - math.log(D) / 2).requires_grad_()
    ang = torch.rand(N, D // 2, generator=g, device="cuda") * 3
    return x, w, rw, sc, ang.sin(), ang.cos()


def _ok(result):
    assert set(result.values()) == {"SUCCESS"}, result


def test_opcheck_inverse_ops():
    q, k, w, s, sin, cos = _prologue_args()
    _ok(torch.library.opcheck(OPS.qknorm_rope_scale_cute_inverse.default, (q, k, w, s, sin, cos, 1e-5),
                              test_utils=CHECKS))
    qo, ko, rq, rk = OPS.qknorm_rope_scale_cute_inverse(q, k, w, s, sin, cos, 1e-5)
    g = torch.randn_like(qo)
    _ok(torch.library.opcheck(OPS.qknorm_rope_scale_cute_inverse_backward.default,
                              (qo.detach(), ko.detach(), w.detach(), s.detach(), sin, cos, g, g,
                               rq.detach(), rk.detach(), 1e-5), test_utils=CHECKS))


def test_opcheck_qkv_backward_op():
    B, N, H, D = 2, 24, 4, 64
    qkv = torch.randn(B, N, 3, H, D, device="cuda").to(torch.bfloat16)
    _, _, w, s, sin, cos = _prologue_args(B, H, N, D)
    gq = torch.randn(B, H, N, D, device="cuda").to(torch.bfloat16)
    gv = torch.randn(B, N, H, D, device="cuda").to(torch.bfloat16)
    _ok(torch.library.opcheck(OPS.qknorm_rope_scale_qkv_backward.default,
                              (qkv, w.detach(), s.detach(), sin, cos, gq, gq, gv, 1e-5), test_utils=CHECKS))


def test_opcheck_gemm_ops():
    x, w, rw, sc, sin, cos = _gemm_args()
    _ok(torch.library.opcheck(OPS.fused_qkv_epilogue.default, (x, w, rw, sc, sin, cos), test_utils=CHECKS))
    _ok(torch.library.opcheck(OPS.fused_qkv_epilogue_ckp.default, (x, w, rw, sc, sin, cos),
                              test_utils=CHECKS))
    x64, w64, *_ = _gemm_args(D=64, H=4)
    _ok(torch.library.opcheck(OPS.fused_qkv.default, (x64, w64), test_utils=CHECKS))


def test_compiled_packed_qkv_matches_eager():
    T, H, D = 96, 4, 64
    g = torch.Generator(device="cuda").manual_seed(4)
    qkv = torch.randn(T, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    ang = torch.rand(T, D // 2, generator=g, device="cuda") * 3
    sin, cos = ang.sin(), ang.cos()
    grads = [torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3)]

    def step(fn):
        x = qkv.detach().clone().requires_grad_()
        wl, sl = w.detach().clone().requires_grad_(), s.detach().clone().requires_grad_()
        outs = fn(x, wl, sl, sin, cos)
        return outs, torch.autograd.grad(outs, (x, wl, sl), grads)

    eager = step(fap.qknorm_rope_scale_qkv)
    compiled = step(torch.compile(fap.qknorm_rope_scale_qkv, fullgraph=True, dynamic=False))
    for a, b in zip(eager[0] + eager[1], compiled[0] + compiled[1]):
        assert torch.equal(a, b)


def test_compiled_fused_qkv_epilogue_matches_eager():
    x, w, rw, sc, sin, cos = _gemm_args(N=256)
    grads = [torch.randn(1, 2, 256, 128, device="cuda").to(torch.bfloat16) for _ in range(3)]

    def fn(*a):
        return fap.fused_qkv_epilogue(*a)[:3]

    def step(f):
        leaves = [t.detach().clone().requires_grad_(i < 4) for i, t in enumerate((x, w, rw, sc, sin, cos))]
        outs = f(*leaves)
        return outs, torch.autograd.grad(outs, leaves[:4], grads)

    eager = step(fn)
    compiled = step(torch.compile(fn, fullgraph=True, dynamic=False))
    for a, b in zip(eager[0] + eager[1], compiled[0] + compiled[1]):
        assert torch.equal(a, b)


def test_opcheck_reference_qkv_op():
    from flash_attn_prologue_b200 import epilogue_kernel  # noqa: F401  (registers the op)
    B, N, H, D = 2, 24, 4, 64
    qkv = torch.randn(B, N, 3 * H * D, device="cuda").to(torch.bfloat16).requires_grad_()
    _, _, w, s, sin, cos = _prologue_args(B, H, N, D)
    _ok(torch.library.opcheck(OPS.qknorm_rope_scale.default, (qkv, w, s, sin, cos, 1e-5), test_utils=CHECKS))
