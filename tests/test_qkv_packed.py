"""qknorm_rope_scale_qkv: the prologue on the Q/K slots of a fused QKV activation.

CPU: the ``native`` path equals the reference frontend on the unbound slices
(flash_attn_prologue/functional.py:14-94). GPU: the ``cute`` path's outputs
are bit-identical to qknorm_rope_scale on the slice views, and its single
gradient tensor equals, bit for bit, the gradient autograd gathers from the
slice views (dq, dk from the same kernel; dv in the V slot; zeros when v is
unused); the parameter gradients are identical too.
"""
import math

import pytest
import torch

import flash_attn_prologue_b200 as fap


def _problem(shape, dtype=torch.bfloat16, seed=0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    H, D = shape[-2], shape[-1]
    qkv = torch.randn(shape, generator=g).to(dtype)
    w = 1 + 0.2 * torch.randn(2, 1, D, generator=g)
    s = 0.2 * torch.randn(H, 1, 1, generator=g) - math.log(D) / 2
    n = shape[0] if len(shape) == 4 else shape[1]
    ang = torch.rand(n, D // 2, generator=g) * 6.0
    return [t.to(device) for t in (qkv, w, s, ang.sin(), ang.cos())]


def _slices(qkv):
    q, k, v = qkv.unbind(-3)
    if qkv.ndim == 5:
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    return q, k, v


@pytest.mark.parametrize("shape", [(37, 3, 4, 32), (2, 19, 3, 2, 64)])
def test_native_path_matches_frontend_on_slices(shape):
    qkv, w, s, sin, cos = _problem(shape)
    q_out, k_out, v = fap.qknorm_rope_scale_qkv(qkv, w, s, sin, cos, backend="native")
    q, k, v_ref = _slices(qkv)
    rq, rk = fap.qknorm_rope_scale(q, k, w, s, sin, cos, backend="native")
    assert torch.equal(q_out, rq) and torch.equal(k_out, rk) and torch.equal(v, v_ref)


def test_rejects_bad_qkv_shapes():
    qkv, w, s, sin, cos = _problem((8, 3, 2, 32))
    with pytest.raises(ValueError):
        fap.qknorm_rope_scale_qkv(qkv[:, :2], w, s, sin, cos, backend="native")
    with pytest.raises(ValueError):
        fap.qknorm_rope_scale_qkv(qkv[0], w, s, sin, cos, backend="native")
    with pytest.raises(ValueError, match="FP32"):
        fap.qknorm_rope_scale_qkv(qkv, w.double(), s, sin, cos, backend="native")


def _grads_via_slices(qkv, w, s, sin, cos, gq, gk, gv):
    x = qkv.detach().clone().requires_grad_()
    wl, sl = w.detach().clone().requires_grad_(), s.detach().clone().requires_grad_()
    q, k, v = _slices(x)
    q_out, k_out = fap.qknorm_rope_scale(q, k, wl, sl, sin, cos, backend="cute")
    outs, grads = (q_out, k_out), (gq, gk)
    if gv is not None:
        outs, grads = outs + (v,), grads + (gv,)
    return (q_out, k_out, v), torch.autograd.grad(outs, (x, wl, sl), grads)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1000, 3, 16, 64), (3, 77, 3, 4, 128), (513, 3, 8, 32)])
@pytest.mark.parametrize("use_v", [True, False])
def test_cute_gradient_equals_gathered_slice_gradients(shape, use_v):
    qkv, w, s, sin, cos = _problem(shape, seed=len(shape) + shape[-1], device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    gq, gk, gv = (torch.randn(_slices(qkv)[0].shape, generator=g, device="cuda").to(qkv.dtype)
                  for _ in range(3))
    gv = gv if use_v else None
    ref_outs, ref_grads = _grads_via_slices(qkv, w, s, sin, cos, gq, gk, gv)
    x = qkv.detach().clone().requires_grad_()
    wl, sl = w.detach().clone().requires_grad_(), s.detach().clone().requires_grad_()
    q_out, k_out, v = fap.qknorm_rope_scale_qkv(x, wl, sl, sin, cos)
    assert torch.equal(q_out, ref_outs[0]) and torch.equal(k_out, ref_outs[1])
    assert torch.equal(v, ref_outs[2]) and v.data_ptr() == x[..., 2, :, :].data_ptr()
    outs, grads = (q_out, k_out), (gq, gk)
    if gv is not None:
        outs, grads = outs + (v,), grads + (gv,)
    got = torch.autograd.grad(outs, (x, wl, sl), grads)
    torch.cuda.synchronize()
    for a, b in zip(got, ref_grads):
        assert a.shape == b.shape and torch.equal(a, b)
    if gv is None:
        assert float(got[0][..., 2, :, :].abs().max()) == 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1000, 3, 16, 64), (3, 77, 3, 4, 128), (513, 3, 8, 32),
                                   (4096, 3, 16, 64)])
@pytest.mark.parametrize("use_v", [True, False])
def test_cute_packed_gradient_matches_oracle(shape, use_v):
    """The packed path against the CPU oracle directly (not against another CUDA path).

    Outputs: 1 BF16 ulp or the FP32 rounding band of a near-cancelling rotation
    (oracle.check_outputs), > 99% bit-exact. The one gradient tensor: its Q/K
    slots hold dq/dk within the reference suite's BF16 tolerance and 5e-3
    relative L2 error of the oracle's autograd gradients; its V slot holds the
    upstream dv bit for bit (zeros when v is unused); d rmsnorm_weight and
    d scales within 1e-3 relative error. The reference returns compact
    gradients of the slices (flash_attn_prologue/fused_epilogue.py:1401-1402);
    their values are what the slots must hold.
    """
    from oracle import check_outputs, native_forward_backward, term_magnitudes
    from tests._util import rel_err
    qkv, w, s, sin, cos = _problem(shape, seed=len(shape) * 11 + shape[-1] + shape[-2])
    g = torch.Generator().manual_seed(17)
    q, k, _ = _slices(qkv)
    gq, gk, gv = (torch.randn(q.shape, generator=g).to(qkv.dtype) for _ in range(3))
    ref_out, ref_grads = native_forward_backward(q, k, w, s, sin, cos, gq, gk)

    x = qkv.cuda().requires_grad_()
    wl, sl = w.cuda().requires_grad_(), s.cuda().requires_grad_()
    q_out, k_out, v = fap.qknorm_rope_scale_qkv(x, wl, sl, sin.cuda(), cos.cuda())
    outs, ups = (q_out, k_out), (gq.cuda(), gk.cuda())
    if use_v:
        outs, ups = outs + (v,), ups + (gv.cuda(),)
    dqkv, dw, ds = torch.autograd.grad(outs, (x, wl, sl), ups)
    torch.cuda.synchronize()

    for got, exp, mag in zip((q_out, k_out), ref_out, term_magnitudes(q, k, w, s, sin, cos)):
        ok, stats = check_outputs(got.cpu(), exp, mag)
        assert ok and stats["exact_frac"] > 0.99, stats
    dq, dk, dv = _slices(dqkv.cpu())
    for got, exp, nm in ((dq, ref_grads[0], "dq"), (dk, ref_grads[1], "dk")):
        torch.testing.assert_close(got.float(), exp.float(), rtol=1e-2, atol=1e-2, msg=nm)
        assert rel_err(got, exp) < 5e-3, nm
    assert torch.equal(dv, gv if use_v else torch.zeros_like(gv))
    assert rel_err(dw.cpu(), ref_grads[2]) < 1e-3
    assert rel_err(ds.cpu(), ref_grads[3]) < 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("weight_2d", [False, True])
def test_reference_qkv_op_matches_slice_path(weight_2d):
    """flash_prologue::qknorm_rope_scale on [B, N, 3*H*D] (reference epilogue_kernel.py:247-369):
    outputs and gradients equal to the frontend on the slices (the same kernels)."""
    B, N, H, D = 2, 40, 4, 64
    g = torch.Generator(device="cuda").manual_seed(8)
    qkv = torch.randn(B, N, 3 * H * D, generator=g, device="cuda").to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    ang = torch.rand(N, D // 2, generator=g, device="cuda") * 3
    sin, cos = ang.sin()[None, None], ang.cos()[None, None]
    gq, gk, gv = (torch.randn(B, H, N, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    x = qkv.detach().clone().requires_grad_()
    wl = (w[:, 0] if weight_2d else w).detach().clone().requires_grad_()
    sl = s.detach().clone().requires_grad_()
    q, k, v = fap.qknorm_rope_scale_op(x, wl, sl, sin, cos, 1e-5)
    assert q.is_contiguous() and v.is_contiguous() and q.shape == (B, H, N, D)
    got = torch.autograd.grad((q, k, v), (x, wl, sl), (gq, gk, gv))
    xr = qkv.detach().clone().requires_grad_()
    wr, sr = w.detach().clone().requires_grad_(), s.detach().clone().requires_grad_()
    qs, ks, vs = xr.view(B, N, 3, H, D).unbind(2)
    rq, rk = fap.qknorm_rope_scale(qs.transpose(1, 2), ks.transpose(1, 2), wr, sr, sin, cos, backend="cute")
    ref = torch.autograd.grad((rq, rk, vs.transpose(1, 2)), (xr, wr, sr), (gq, gk, gv))
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, vs.transpose(1, 2))
    assert torch.equal(got[0], ref[0])
    assert torch.equal(got[1], ref[1].reshape(got[1].shape)) and torch.equal(got[2], ref[2])
