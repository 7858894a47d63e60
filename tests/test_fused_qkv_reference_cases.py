"""The reference's fused QKV + epilogue tests at their own shapes and tolerances.

tests/test_fused_qkv_epilogue.py of the reference: B = 32, N = 512, hidden =
512, H = 16, D = 64, x / weight / rmsnorm_weight / scales ~ N(0, 1), dense
sin/cos [B, 1, N, D/2] (theta 10000). The sequential chain ``fused_qkv`` ->
``qknorm_rope_scale_cute`` and the fused ``fused_qkv_epilogue`` (and
``fused_qkv_epilogue_ckp``), both under torch.compile (inductor), must agree
on outputs (rtol 1e-2, atol 1e-1) and on the gradients of x, weight,
rmsnorm_weight (rtol 1e-2, atol 1e-1) and scales (rtol 1e-2, atol 6.0).
"""
import pytest
import torch

import flash_attn_prologue_b200 as fap
from flash_attn_prologue_b200 import prepare_backend

fap.fused_qkv_epilogue  # noqa: B018  (the lazy export loads and registers the fused QKV ops)

pytestmark = pytest.mark.gpu
OPS = torch.ops.flash_prologue
B, N, HIDDEN, H, D = 32, 512, 512, 16, 64


def _inputs():
    torch.manual_seed(0)
    x = torch.randn(B, N, HIDDEN, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3 * H * D, HIDDEN, device="cuda", dtype=torch.bfloat16)
    rw = torch.randn(2, 1, D, device="cuda")
    sc = torch.randn(H, 1, 1, device="cuda")
    pos = torch.arange(N, device="cuda").float()[None].expand(B, N)
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    f = torch.outer(pos.reshape(-1), inv).reshape(B, N, -1)
    return x, w, rw, sc, f.sin()[:, None].contiguous(), f.cos()[:, None].contiguous()


def _sequential(x, w, rw, sc, sin, cos):
    q, k, v = OPS.fused_qkv(x, w)
    qo, ko = OPS.qknorm_rope_scale_cute(q, k, rw, sc, sin, cos)
    return qo, ko, v


def _fused(x, w, rw, sc, sin, cos):
    q, k, v, _, _ = OPS.fused_qkv_epilogue(x, w, rw, sc, sin, cos)
    return q, k, v


def _fused_ckp(x, w, rw, sc, sin, cos):
    return OPS.fused_qkv_epilogue_ckp(x, w, rw, sc, sin, cos)


def _run(fn, inputs):
    leaves = [t.clone().detach().requires_grad_() for t in inputs[:4]]
    out = torch.compile(fn, backend="inductor")(*leaves, *inputs[4:])
    (out[0].sum() + out[1].sum() + out[2].sum()).backward()
    return out, [t.grad for t in leaves]


@pytest.mark.parametrize("combined", [_fused, _fused_ckp], ids=["epilogue", "ckp"])
def test_combined_matches_sequential_chain_under_compile(combined):
    prepare_backend("cute")
    inputs = _inputs()
    out_s, grads_s = _run(_sequential, inputs)
    out_c, grads_c = _run(combined, inputs)
    torch.cuda.synchronize()
    for a, b in zip(out_c, out_s):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-1)
    for a, b in zip(grads_c[:3], grads_s[:3]):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-1)
    torch.testing.assert_close(grads_c[3], grads_s[3], rtol=1e-2, atol=6.0)
