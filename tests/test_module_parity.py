"""RMSNormRoPEScale module parity, as the reference's tests/test_fused_epilogue_module.py.

B = 32, H = 16, D = 64, N in {64, 100, 128, 512}; dense sin/cos [B, 1, N, D/2]
(theta 10000); BF16 activations with FP32 master parameters; outputs and input
gradients against an eager FP32 formulation with split-half RoPE, at the
reference test's tolerances (rtol 1e-2, atol 1e-1), eager and under
torch.compile(fullgraph=True). The reference test runs the module's default
backend (native); both backends are run here.
"""
import pytest
import torch

from flash_attn_prologue_b200 import RMSNormRoPEScale

pytestmark = pytest.mark.gpu
B, H, D = 32, 16, 64


def _rope(x, sin, cos):
    """Split-half rotation in FP32, as the reference's layers/RoPE.py apply_rope."""
    x1, x2 = x.float().chunk(2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)


def _tables(N):
    pos = torch.arange(N, device="cuda").unsqueeze(0).expand(B, N).float()
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float32, device="cuda") / D))
    freqs = torch.outer(pos.reshape(-1), inv_freq).reshape(B, N, -1)
    return freqs.sin().unsqueeze(1).contiguous(), freqs.cos().unsqueeze(1).contiguous()


@pytest.mark.parametrize("compiled", [False, True])
@pytest.mark.parametrize("backend", ["native", "cute"])
@pytest.mark.parametrize("N", [64, 100, 128, 512])
def test_module_parity(N, backend, compiled):
    torch.manual_seed(N)
    module = RMSNormRoPEScale(num_heads=H, head_dim=D, backend=backend).to(device="cuda", dtype=torch.bfloat16)
    assert module.rmsnorm_weight.dtype == torch.float32 and module.scales.dtype == torch.float32
    fn = torch.compile(module, fullgraph=True) if compiled else module
    q = torch.randn(B, H, N, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, H, N, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    sin, cos = _tables(N)
    q_ref, k_ref = (t.detach().clone().requires_grad_() for t in (q, k))
    q_out, k_out = fn(q, k, sin, cos)
    eps = module.eps
    qn = q_ref.float() * torch.rsqrt(q_ref.float().pow(2).mean(-1, keepdim=True) + eps) * module.rmsnorm_weight[0, 0]
    kn = k_ref.float() * torch.rsqrt(k_ref.float().pow(2).mean(-1, keepdim=True) + eps) * module.rmsnorm_weight[1, 0]
    q_expect = (_rope(qn, sin, cos) * module.scales.float().exp()).to(torch.bfloat16)
    k_expect = _rope(kn, sin, cos).to(torch.bfloat16)
    torch.testing.assert_close(q_out, q_expect, rtol=1e-2, atol=1e-1)
    torch.testing.assert_close(k_out, k_expect, rtol=1e-2, atol=1e-1)
    (q_out.sum() + k_out.sum()).backward()
    (q_expect.sum() + k_expect.sum()).backward()
    torch.testing.assert_close(q.grad, q_ref.grad, rtol=1e-2, atol=1e-1)
    torch.testing.assert_close(k.grad, k_ref.grad, rtol=1e-2, atol=1e-1)
