"""The ops inside CUDA graphs: capture forward + backward once, replay with new inputs.

A captured step must reproduce the eager results bit for bit after its
static input buffers are refilled (the library launches on the capturing
stream, allocates nothing itself and keeps no per-call host state that a
replay would miss).
"""
import pytest
import torch

import flash_attn_prologue_b200 as fap

pytestmark = pytest.mark.gpu


def _inputs(T=4096, H=4, D=32, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    ang = torch.rand(T, D // 2, generator=g, device="cuda") * 6
    gq = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    gk = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    return q, k, w, s, ang.sin(), ang.cos(), gq, gk


def _step(q, k, w, s, sin, cos, gq, gk):
    qq, kk = q.detach().requires_grad_(), k.detach().requires_grad_()
    ww, ss = w.detach().requires_grad_(), s.detach().requires_grad_()
    out = fap.qknorm_rope_scale(qq, kk, ww, ss, sin, cos, backend="cute")
    grads = torch.autograd.grad(out, (qq, kk, ww, ss), (gq, gk))
    return (*out, *grads)


@pytest.mark.parametrize("T,H,D", [(4096, 4, 32), (8192, 16, 64)])
def test_captured_fwd_bwd_replays_like_eager(T, H, D):
    fap.prepare_backend("cute")
    static = _inputs(T, H, D, seed=1)
    for _ in range(2):  # warm up the allocator and the library's one-time setup
        _step(*static)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = _step(*static)
    for seed in (2, 3):
        fresh = _inputs(T, H, D, seed=seed)
        for dst, src in zip(static, fresh):
            dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize()
        eager = _step(*fresh)
        for a, b in zip(captured, eager):
            assert torch.equal(a, b)
