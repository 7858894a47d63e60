"""Inverse (recompute-from-outputs) prologue ops on the GPU, through the C ABI.

``flash_prologue::qknorm_rope_scale_cute_inverse`` must return exactly the
outputs of the regular forward plus r = 1/sqrt(mean(x^2)+eps) per row (within
the FP32 rounding of the D-term sum of squares, relative 2e-6, of the oracle's); ``..._inverse_backward`` is checked
against the oracle's restatement of the reference's inverse backward
(oracle/inverse.py) fed the same outputs and statistics: dq/dk within 1 ulp of
the activation dtype for > 99% of elements and 2e-3 relative L2 error overall,
d rmsnorm_weight / d scales within 1e-3 relative error. The reference's own
test (tests/test_fused_epilogue_inverse.py) runs as written, tolerances included.
Reference: flash_attn_prologue/fused_epilogue.py:2560-2805.
"""
import math

import pytest
import torch

import flash_attn_prologue_b200  # noqa: F401  (registers the ops)
from flash_attn_prologue_b200 import _lib, fused_epilogue  # noqa: F401
from oracle import inverse_backward, inverse_forward
from tests._util import rel_err, ulp_diff

pytestmark = pytest.mark.gpu

OPS = torch.ops.flash_prologue


def _problem(B, H, N, D, dtype=torch.bfloat16, seed=0, batch_tables=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g).to(dtype)
    k = torch.randn(B, H, N, D, generator=g).to(dtype)
    w = 1 + 0.2 * torch.randn(2, 1, D, generator=g)
    s = 0.2 * torch.randn(H, 1, 1, generator=g) - math.log(D) / 2
    pos = torch.arange(N, dtype=torch.float64)
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = (pos[:, None] * inv[None]).float()[None, None]
    if batch_tables:
        ang = ang + 0.01 * torch.arange(B, dtype=torch.float32).reshape(B, 1, 1, 1)
    gq = torch.randn(B, H, N, D, generator=g).to(dtype)
    gk = torch.randn(B, H, N, D, generator=g).to(dtype)
    return q, k, w, s, ang.sin(), ang.cos(), gq, gk


def _check_inverse(q, k, w, s, sin, cos, gq, gk, eps=1e-5):
    """Runs both inverse ops on the given CUDA views and checks them against the oracle."""
    q_out, k_out, rms_q, rms_k = OPS.qknorm_rope_scale_cute_inverse(q, k, w, s, sin, cos, eps)
    ref_q, ref_k = OPS.qknorm_rope_scale_cute(q, k, w, s, sin, cos, eps)
    torch.cuda.synchronize()
    assert _lib.device_error(reset=True) == 0
    # Outputs: bit-identical to the regular forward.
    assert torch.equal(q_out, ref_q) and torch.equal(k_out, ref_k)
    assert q_out.stride() == ref_q.stride()
    assert rms_q.shape == (*q.shape[:3], 1) and rms_q.dtype == torch.float32
    cpu = [t.cpu() for t in (q, k, w, s, sin, cos)]
    _, _, oq, ok = inverse_forward(*cpu, eps=eps)
    for got, exp in ((rms_q, oq), (rms_k, ok)):
        torch.testing.assert_close(got.cpu(), exp, rtol=2e-6, atol=0)
    dq, dk, dw, ds = OPS.qknorm_rope_scale_cute_inverse_backward(
        q_out, k_out, w, s, sin, cos, gq, gk, rms_q, rms_k, eps)
    torch.cuda.synchronize()
    assert _lib.device_error(reset=True) == 0
    rdq, rdk, rdw, rds = inverse_backward(q_out.cpu(), k_out.cpu(), w.cpu(), s.cpu(), sin.cpu(),
                                          cos.cpu(), gq.cpu(), gk.cpu(), rms_q.cpu(), rms_k.cpu())
    for got, exp, nm in ((dq, rdq, "dq"), (dk, rdk, "dk")):
        got = got.cpu()
        assert got.dtype == exp.dtype and got.shape == exp.shape, nm
        if got.dtype == torch.float32:
            assert rel_err(got, exp) < 1e-5, nm
        else:
            d = ulp_diff(got.contiguous(), exp.contiguous())
            assert float((d <= 1).float().mean()) > 0.99, (nm, int(d.max()))
            assert rel_err(got, exp) < 2e-3, nm
    assert rel_err(dw.cpu(), rdw) < 1e-3, "dw"
    assert rel_err(ds.cpu(), rds) < 1e-3, "ds"
    return (q_out, k_out, rms_q, rms_k), (dq, dk, dw, ds)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_dense_dims_dtypes(D, dtype):
    args = [t.cuda() for t in _problem(2, 4, 67, D, dtype, seed=D)]
    _check_inverse(*args)


@pytest.mark.parametrize("H", [1, 3, 5])
@pytest.mark.parametrize("D", [64, 128])
def test_odd_head_counts_every_path(H, D):
    """Odd head counts on every kernel path (automatic, register path, TMA-stored
    and lane-stored outputs). The per-head arrays in the backward's shared memory
    then have odd lengths, and the float-pair reads of w and 1/w must stay
    8-byte aligned; every path gives the same bits and matches the oracle."""
    args = [t.cuda() for t in _problem(2, H, 77, D, seed=30 + H + D)]
    results = []
    try:
        for mode in (0, 1, 2, 3):
            _lib.set_path(mode)
            results.append(_check_inverse(*args))
    finally:
        _lib.set_path(0)
    (f0, g0) = results[0]
    for mode, (f, g) in zip((1, 2, 3), results[1:]):
        for x, y in zip(f0 + g0[:2], f + g[:2]):
            assert torch.equal(x, y), mode
        for x, y in zip(g0[2:], g[2:]):
            assert rel_err(x, y) < 1e-5, mode


def test_packed_strided_qkv_views_both_paths():
    """q = buf[:, 0], k = buf[:, 1] of a [T, 3, H, D] buffer, as [1, H, T, D] views."""
    T, H, D = 1000, 16, 64
    g = torch.Generator().manual_seed(7)
    buf = torch.randn(T, 3, H, D, generator=g).to(torch.bfloat16).cuda()
    q = buf[:, 0].permute(1, 0, 2)[None]
    k = buf[:, 1].permute(1, 0, 2)[None]
    _, _, w, s, sin, cos, gq, gk = (t.cuda() for t in _problem(1, H, T, D, seed=8))
    results = []
    try:
        for mode in (0, 1):  # TMA pipeline, register path
            _lib.set_path(mode)
            results.append(_check_inverse(q, k, w, s, sin, cos, gq, gk))
    finally:
        _lib.set_path(0)
    (fa, ga), (fb, gb) = results
    for x, y in zip(fa + ga[:2], fb + gb[:2]):
        assert torch.equal(x, y)  # same per-row arithmetic on both paths
    for x, y in zip(ga[2:], gb[2:]):
        assert rel_err(x, y) < 1e-5  # fixed-order sums over different grids


def test_misaligned_views_and_batch_tables():
    B, H, N, D = 3, 2, 50, 64
    q, k, w, s, sin, cos, gq, gk = _problem(B, H, N, D, seed=11, batch_tables=True)
    base = torch.zeros(q.numel() + 8, dtype=q.dtype).cuda()
    qm = base[1:1 + q.numel()].view(q.shape).copy_(q)  # 2-byte offset: register path
    _check_inverse(qm, k.cuda(), w.cuda(), s.cuda(), sin.cuda(), cos.cuda(), gq.cuda(), gk.cuda())


def test_eps_is_honoured():
    args = [t.cuda() for t in _problem(1, 2, 33, 64, seed=12)]
    args[0] = args[0] * 0.01  # small rows: eps dominates
    _check_inverse(*args, eps=0.1)


def test_autograd_through_inverse_op():
    q, k, w, s, sin, cos, gq, gk = (t.cuda() for t in _problem(2, 4, 40, 64, seed=13))
    leaves = [t.clone().requires_grad_() for t in (q, k, w, s)]
    q_out, k_out, rms_q, rms_k = OPS.qknorm_rope_scale_cute_inverse(*leaves, sin, cos, 1e-5)
    grads = torch.autograd.grad((q_out, k_out), leaves, (gq, gk))
    direct = OPS.qknorm_rope_scale_cute_inverse_backward(q_out.detach(), k_out.detach(), w, s, sin, cos,
                                                         gq, gk, rms_q.detach(), rms_k.detach(), 1e-5)
    for a, b in zip(grads, direct):
        assert torch.equal(a, b)
    # Only one output used: the other's gradient is zero.
    q_out, _, _, _ = OPS.qknorm_rope_scale_cute_inverse(*leaves, sin, cos, 1e-5)
    dq, dk = torch.autograd.grad(q_out, leaves[:2], gq)
    assert float(dk.abs().max()) == 0.0


def test_empty_inputs():
    q, k, w, s, sin, cos, _, _ = (t.cuda() for t in _problem(2, 4, 1, 64))
    qe, ke = q[:, :, :0], k[:, :, :0]
    out = OPS.qknorm_rope_scale_cute_inverse(qe, ke, w, s, sin[:, :, :0], cos[:, :, :0], 1e-5)
    assert out[0].shape == qe.shape and out[2].shape == (2, 4, 0, 1)
    dq, dk, dw, ds = OPS.qknorm_rope_scale_cute_inverse_backward(
        out[0], out[1], w, s, sin[:, :, :0], cos[:, :, :0], out[0], out[1], out[2], out[3], 1e-5)
    assert dq.shape == qe.shape and float(dw.abs().sum()) == 0.0 and float(ds.abs().sum()) == 0.0


def test_reference_suite_inverse_correctness():
    """The reference's tests/test_fused_epilogue_inverse.py, shapes and tolerances as written
    (BF16 parameters; eager baseline with the reference's FP32 split-half RoPE)."""
    B, N, H, D, eps = 4, 128, 4, 64, 1e-5
    dtype, device = torch.bfloat16, "cuda"
    torch.manual_seed(0)
    w = torch.nn.Parameter(torch.ones(2, 1, D, device=device, dtype=dtype))
    s = torch.nn.Parameter(torch.full((H, 1, 1), -2.0, device=device, dtype=dtype))
    q = torch.randn(B, H, N, D, device=device, dtype=dtype, requires_grad=True)
    k = torch.randn(B, H, N, D, device=device, dtype=dtype, requires_grad=True)
    pos = torch.arange(N, device=device).unsqueeze(0).expand(B, N).float()
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float32, device=device) / D))
    freqs = torch.outer(pos.reshape(-1), inv_freq).reshape(B, N, -1)
    sin = torch.sin(freqs).unsqueeze(1).contiguous()
    cos = torch.cos(freqs).unsqueeze(1).contiguous()

    def clones():
        return [t.clone().detach().requires_grad_(True) for t in (q, k, w, s)]

    qr, kr, wr, sr = clones()
    qn = qr.float() * torch.rsqrt(qr.float().pow(2).mean(-1, keepdim=True) + eps) * wr[0, 0].float()
    kn = kr.float() * torch.rsqrt(kr.float().pow(2).mean(-1, keepdim=True) + eps) * wr[1, 0].float()

    def rope(x):  # the reference's layers/RoPE.py apply_rope: FP32 rotation, cast back
        x1, x2 = x.float().chunk(2, dim=-1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)

    q_ref = rope(qn.to(dtype)) * sr.float().exp().to(dtype)
    k_ref = rope(kn.to(dtype))
    qs, ks, ws, ss = clones()
    q_std, k_std = OPS.qknorm_rope_scale_cute(qs, ks, ws, ss, sin, cos, eps)
    qi, ki, wi, si = clones()
    q_inv, k_inv, _, _ = OPS.qknorm_rope_scale_cute_inverse(qi, ki, wi, si, sin, cos, eps)
    for got in (q_std, q_inv):
        torch.testing.assert_close(got, q_ref, rtol=1e-2, atol=1e-1)
    for got in (k_std, k_inv):
        torch.testing.assert_close(got, k_ref, rtol=1e-2, atol=1e-1)
    (q_ref.sum() + k_ref.sum()).backward()
    (q_std.sum() + k_std.sum()).backward()
    (q_inv.sum() + k_inv.sum()).backward()
    torch.testing.assert_close(qi.grad, qs.grad, rtol=1e-2, atol=2e-1)
    torch.testing.assert_close(ki.grad, ks.grad, rtol=1e-2, atol=2e-1)
    torch.testing.assert_close(qi.grad, qr.grad, rtol=1e-2, atol=2e-1)
    torch.testing.assert_close(ki.grad, kr.grad, rtol=1e-2, atol=2e-1)
    torch.testing.assert_close(wi.grad, ws.grad, rtol=1e-2, atol=2.5e-1)
    torch.testing.assert_close(wi.grad, wr.grad, rtol=1e-2, atol=5e-1)
    torch.testing.assert_close(si.grad, ss.grad, rtol=1e-2, atol=2e-1)
    torch.testing.assert_close(si.grad, sr.grad, rtol=1e-2, atol=3e-1)


def test_full_size_c2_inverse_sampled_rows():
    """C2 shape (T = 1,048,576, H = 16, D = 64) from a [T, 3, H, D] buffer; sampled rows vs oracle."""
    T, H, D = 1 << 20, 16, 64
    g = torch.Generator(device="cuda").manual_seed(21)
    buf = torch.randn(T, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
    q = buf[:, 0].permute(1, 0, 2)[None]
    k = buf[:, 1].permute(1, 0, 2)[None]
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    pos = (torch.arange(T, device="cuda") % 4096).double()
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float64) / D))
    ang = (pos[:, None] * inv[None]).float()
    sin, cos = ang.sin()[None, None], ang.cos()[None, None]
    gq = torch.randn(1, H, T, D, generator=g, device="cuda").to(torch.bfloat16)
    gk = torch.randn(1, H, T, D, generator=g, device="cuda").to(torch.bfloat16)
    q_out, k_out, rms_q, rms_k = OPS.qknorm_rope_scale_cute_inverse(q, k, w, s, sin, cos, 1e-5)
    dq, dk, dw, ds = OPS.qknorm_rope_scale_cute_inverse_backward(q_out, k_out, w, s, sin, cos, gq, gk,
                                                                rms_q, rms_k, 1e-5)
    torch.cuda.synchronize()
    assert _lib.device_error(reset=True) == 0
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:2048].cuda()
    pick = lambda t: t[:, :, idx].cpu()  # noqa: E731
    rdq, rdk, _, _ = inverse_backward(pick(q_out), pick(k_out), w.cpu(), s.cpu(), pick(sin), pick(cos),
                                      pick(gq), pick(gk), pick(rms_q), pick(rms_k))
    for got, exp in ((pick(dq), rdq), (pick(dk), rdk)):
        d = ulp_diff(got.contiguous(), exp.contiguous())
        assert float((d <= 1).float().mean()) > 0.99 and rel_err(got, exp) < 2e-3
    # Parameter gradients over all rows: FP32 torch formulation of the same identities.
    _, _, rdw, rds = inverse_backward(q_out, k_out, w, s, sin, cos, gq, gk, rms_q, rms_k)
    assert rel_err(dw, rdw) < 1e-3 and rel_err(ds, rds) < 1e-3
