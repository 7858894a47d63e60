"""Fused QKV projection GEMM (tcgen05/TMEM) with the prologue in its epilogue.

Parity is checked in two parts, so each has its own bar:
* the projection: against X.float() @ W.float().T rounded to BF16 (both
  accumulate in FP32; only the order differs) -- within 1 BF16 ulp, except
  where the dot product cancels, where the error must stay within 2^-20 of
  sum_k |x_k w_k| (FP32 rounding of the terms); > 99.9% within 1 ulp;
* the epilogue: Q/K against the oracle's native formulation applied to the
  kernel's own BF16 projections (q_proj/k_proj outputs) -- the prologue bar
  of the other kernels (1 ulp, or the FP32 rounding band of a near-cancelling
  rotation), and V bit-equal to the projection.
Reference semantics: F.linear followed by the native prologue
(flash_attn_prologue/fused_qkv.py:698-878, layers/FusedQKV.py:17-55).
"""
import math

import pytest
import torch

import flash_attn_prologue_b200 as fap
from oracle import check_outputs, native_forward, term_magnitudes
from tests._util import rel_err, ulp_diff

pytestmark = pytest.mark.gpu


def _problem(B, N, hidden, H, D, seed=0, theta=10000.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, N, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(3 * H * D, hidden, generator=g, device="cuda")).to(torch.bfloat16)
    rw = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    sc = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda") - math.log(D) / 2
    pos = torch.arange(N, device="cuda", dtype=torch.float64)
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float64) / D))
    ang = (pos[:, None] * inv[None]).float()
    return x, w, rw, sc, ang.sin(), ang.cos()


def _split_heads(p, B, N, H, D):
    p = p.reshape(B, N, 3, H, D).permute(2, 0, 3, 1, 4)  # [3, B, H, N, D]
    return p[0], p[1], p[2]


def _projection_reference(x, w, H, D):
    """(BF16 projection, sum |x||w| magnitude) per output, split into heads."""
    B, N, _ = x.shape
    x2 = x.float().reshape(B * N, -1)
    p = (x2 @ w.float().t()).to(torch.bfloat16)
    mag = x2.abs() @ w.float().abs().t()
    return list(zip(_split_heads(p, B, N, H, D), _split_heads(mag, B, N, H, D)))


def _check_projection(got, ref):
    ref, mag = ref
    d = ulp_diff(got.contiguous(), ref.contiguous())
    in_band = (got.float() - ref.float()).abs().cpu() <= (2.0 ** -20) * mag.cpu()
    assert bool(((d <= 1) | in_band).all()), int(d.max())
    assert float((d <= 1).float().mean()) > 0.999


@pytest.mark.parametrize("B,N,hidden,H", [(2, 128, 256, 4), (1, 200, 128, 8), (3, 64, 512, 4)])
def test_gemm_only_matches_fp32_accumulated_projection(B, N, hidden, H):
    x, w, *_ = _problem(B, N, hidden, H, 64, seed=B + N)
    q, k, v = fap.fused_qkv(x, w)
    torch.cuda.synchronize()
    for got, ref in zip((q, k, v), _projection_reference(x, w, H, 64)):
        _check_projection(got, ref)


@pytest.mark.parametrize("D,H", [(128, 2), (128, 4), (64, 4), (64, 8)])
@pytest.mark.parametrize("B,N,hidden", [(2, 128, 256), (1, 200, 192), (2, 64, 1024)])
def test_fused_epilogue_parity(D, H, B, N, hidden):
    x, w, rw, sc, sin, cos = _problem(B, N, hidden, H, D, seed=D * H + N)
    q, k, v, q_proj, k_proj = fap.fused_qkv_epilogue(x, w, rw, sc, sin, cos)
    torch.cuda.synchronize()
    from flash_attn_prologue_b200 import _lib
    assert _lib.device_error(reset=True) == 0
    rq, rk, rv = _projection_reference(x, w, H, D)
    _check_projection(q_proj, rq)
    _check_projection(k_proj, rk)
    _check_projection(v, rv)
    # Epilogue: the native formulation on the kernel's own projections.
    args = (q_proj.cpu(), k_proj.cpu(), rw.cpu(), sc.cpu(), sin.cpu(), cos.cpu())
    ref = native_forward(*args)
    mags = term_magnitudes(*args)
    for got, exp, mag in zip((q, k), ref, mags):
        ok, stats = check_outputs(got.cpu(), exp, mag)
        assert ok and stats["exact_frac"] > 0.99, stats


def test_fused_epilogue_matches_prologue_kernel():
    """The GEMM epilogue and the standalone prologue kernel agree on the same projections."""
    B, N, hidden, H, D = 2, 256, 256, 4, 128
    x, w, rw, sc, sin, cos = _problem(B, N, hidden, H, D, seed=5)
    q, k, _, q_proj, k_proj = fap.fused_qkv_epilogue(x, w, rw, sc, sin, cos)
    q2, k2 = fap.qknorm_rope_scale(q_proj, k_proj, rw, sc, sin, cos, backend="cute")
    args = (q_proj.cpu(), k_proj.cpu(), rw.cpu(), sc.cpu(), sin.cpu(), cos.cpu())
    for a, b, mag in zip((q, k), (q2, k2), term_magnitudes(*args)):
        ok, stats = check_outputs(a.cpu(), b.cpu(), mag)
        assert ok and stats["exact_frac"] > 0.99, stats


def test_fused_epilogue_backward():
    B, N, hidden, H, D = 2, 128, 256, 2, 128
    x, w, rw, sc, sin, cos = _problem(B, N, hidden, H, D, seed=9)
    g = torch.Generator(device="cuda").manual_seed(1)
    gq, gk, gv = (torch.randn(B, H, N, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    a = [t.detach().clone().requires_grad_(i < 4) for i, t in enumerate((x, w, rw, sc, sin, cos))]
    q, k, v, _, _ = fap.fused_qkv_epilogue(*a)
    grads = torch.autograd.grad((q, k, v), a[:4], (gq, gk, gv))
    # Reference: F.linear in FP32 -> BF16 projections -> native prologue, autograd.
    r = [t.detach().clone().float().requires_grad_(i < 4) if i < 2 else t.detach().clone().requires_grad_(i < 4)
         for i, t in enumerate((x, w, rw, sc, sin, cos))]
    p = (r[0].reshape(B * N, hidden) @ r[1].t()).reshape(B, N, 3, H, D).permute(2, 0, 3, 1, 4)
    rq, rk = native_forward(p[0], p[1], r[2], r[3], r[4], r[5])
    rgrads = torch.autograd.grad((rq, rk, p[2]), r[:4], (gq.float(), gk.float(), gv.float()))
    for got, exp in zip(grads, rgrads):
        assert rel_err(got.float(), exp.float()) < 2e-2


def test_rejects_unsupported_shapes():
    x = torch.zeros(1, 8, 100, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(3 * 256, 100, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fap.fused_qkv(x, w)  # hidden not a multiple of 64


def test_config5_full_size_sampled_rows():
    """C5: X [65,536, 2048], W [6144, 2048], H=16, D=128, theta 10000, positions 0..T-1."""
    T, hidden, H, D = 65536, 2048, 16, 128
    x, w, rw, sc, sin, cos = _problem(1, T, hidden, H, D, seed=55)
    q, k, v, q_proj, k_proj = fap.fused_qkv_epilogue(x, w, rw, sc, sin, cos)
    torch.cuda.synchronize()
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:1024].cuda()
    xs = x[0, idx].float()
    p = (xs @ w.float().t()).to(torch.bfloat16).reshape(-1, 3, H, D)
    mag = (xs.abs() @ w.float().abs().t()).reshape(-1, 3, H, D)
    for i, got in enumerate((q_proj, k_proj, v)):
        _check_projection(got[0][:, idx].transpose(0, 1), (p[:, i], mag[:, i]))
    args = (q_proj[0][:, idx].transpose(0, 1).cpu(), k_proj[0][:, idx].transpose(0, 1).cpu(),
            rw.cpu(), sc.cpu(), sin[idx].cpu(), cos[idx].cpu())
    ref = native_forward(*args)
    for got, exp, mag in zip((q[0][:, idx].transpose(0, 1), k[0][:, idx].transpose(0, 1)), ref,
                             term_magnitudes(*args)):
        ok, stats = check_outputs(got.cpu(), exp, mag)
        assert ok and stats["exact_frac"] > 0.99, stats


@pytest.mark.parametrize("B,N,hidden,H,D", [(1, 200, 128, 8, 64), (3, 128, 256, 2, 128),
                                            (1, 1000, 512, 4, 128), (2, 96, 192, 4, 64)])
def test_cta_pair_and_single_cta_mainloops_agree(B, N, hidden, H, D):
    """The 2-CTA (cta_group::2, 256-row tiles) and single-CTA mainloops give identical outputs."""
    from flash_attn_prologue_b200 import _lib
    x, w, rw, sc, sin, cos = _problem(B, N, hidden, H, D, seed=31 + N)
    outs = []
    try:
        for variant in (1, 0):
            _lib.set_gemm_variant(variant)
            outs.append(fap.fused_qkv_epilogue(x, w, rw, sc, sin, cos))
            torch.cuda.synchronize()
            assert _lib.device_error(reset=True) == 0
    finally:
        _lib.set_gemm_variant(0)
    for a, b in zip(*outs):
        assert torch.equal(a, b)
